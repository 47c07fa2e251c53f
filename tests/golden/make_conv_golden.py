#!/usr/bin/env python3
"""Generates tests/golden/convert.json from the REFERENCE's own converters
(gpu-llm/tools/conv_qwen.py and conv_gpt2.py, run unmodified from a
reference checkout) on the seeded synthetic checkpoints of conv_synth.py.

The fixture holds, per model: the seed, the SHA-256 of the synthetic
checkpoint (so a drift of the generator is told apart from a converter
mismatch), and the size plus SHA-256 of the reference's output in 64 MiB
blocks (so a mismatch can be located).

Run from the repository root:
    python tests/golden/make_conv_golden.py [reference checkout]
(default: $SB_REFERENCE_DIR, else the build machine's reference checkout,
the same default as __graft_entry__.build()).  Needs ~4 GB of temporary
space.
"""
import hashlib
import json
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import conv_synth  # noqa: E402

SEEDS = {"qwen": 20261211, "gpt2": 20261212}
BLOCK = 64 << 20


def file_digest(path):
    """(size, whole-file SHA-256, [SHA-256 per 64 MiB block])"""
    whole, blocks, size = hashlib.sha256(), [], 0
    with open(path, "rb") as f:
        while True:
            b = f.read(BLOCK)
            if not b:
                break
            whole.update(b)
            blocks.append(hashlib.sha256(b).hexdigest())
            size += len(b)
    return size, whole.hexdigest(), blocks


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SB_REFERENCE_DIR", "")
    if not ref:
        sys.exit("usage: make_conv_golden.py <reference checkout>  (or set SB_REFERENCE_DIR)")
    tools = os.path.join(ref, "gpu-llm", "tools")
    out = {"block_bytes": BLOCK}
    with tempfile.TemporaryDirectory() as tmp:
        for model, write in (("qwen", conv_synth.write_qwen), ("gpt2", conv_synth.write_gpt2)):
            src = os.path.join(tmp, f"{model}.safetensors")
            dst = os.path.join(tmp, f"{model}.bin")
            write(src, SEEDS[model])
            _, src_sha, _ = file_digest(src)
            script = os.path.join(tools, f"conv_{model}.py")
            r = subprocess.run([sys.executable, script, src, dst], capture_output=True, text=True)
            if r.returncode != 0:
                sys.exit(f"{script} failed ({r.returncode}): {r.stderr[-500:]}")
            size, sha, blocks = file_digest(dst)
            out[model] = {"seed": SEEDS[model], "checkpoint_sha256": src_sha, "bytes": size, "sha256": sha,
                          "block_sha256": blocks}
            print(f"{model}: {size} bytes, {sha}")
            os.unlink(src)
            os.unlink(dst)
    with open(os.path.join(HERE, "convert.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
