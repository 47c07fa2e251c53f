#!/usr/bin/env python3
"""Generates tests/golden/*.json from the REFERENCE's own C (gpu-llm/engine/
{qwen,gpt2}_engine.c compiled unmodified into oracle/_ref/ by
`make -C oracle ref REF=<reference checkout>`).

The fixtures pin the oracle restatement even where oracle/_ref cannot be
built: each holds the reference's outputs on seeded synthetic inputs (the
inputs themselves are regenerated from the stored seeds).  Floats are
stored as float.hex() of the float32 value so comparisons can be exact.

Run from the repository root:  python tests/golden/make_golden.py
"""
import ctypes
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "switch-l4t-gpu_b200"))
sys.path.insert(0, os.path.join(REPO, "tests"))
import conftest  # noqa: E402  (seeds and the synthetic weight files)
import orc  # noqa: E402
import sb200  # noqa: E402


def fhex(a):
    return [float(v).hex() for v in np.asarray(a, dtype=np.float32).ravel()]


def file_digest(path, nbytes=64 << 20):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read(nbytes)).hexdigest()


def logits_record(lg):
    lg = np.asarray(lg, dtype=np.float32)
    top = np.argsort(-lg, kind="stable")[:5]
    return {"argmax": int(np.argmax(lg)), "top5": [int(i) for i in top], "first16": fhex(lg[:16]),
            "sum": float(lg.astype(np.float64).sum()), "sumsq": float((lg.astype(np.float64) ** 2).sum()),
            "sha256": hashlib.sha256(lg.tobytes()).hexdigest()}


def engine_fixture(name, path, seed, vocab, n_tok, id_seed):
    L = orc.ref_lib(name)
    getattr(L, f"ref_{name}_load")(path.encode())
    ids = sb200.synth_ids(n_tok, vocab, id_seed)
    steps = []
    lg = np.zeros(vocab, dtype=np.float32)
    for p, t in enumerate(ids):
        getattr(L, f"ref_{name}_forward")(t, p, 1, lg.ctypes.data_as(ctypes.c_void_p))
        steps.append(logits_record(lg))
    return {"model": name, "weights_seed": seed, "weights_sha256_first64MiB": file_digest(path),
            "ids_seed": id_seed, "ids": ids, "steps": steps,
            "source": f"gpu-llm/engine/{name}_engine.c cpu_forward (reference, unmodified)"}


def gemv_h_fixture():
    L = orc.ref_lib("qwen")
    rng = np.random.default_rng(1)
    N, K = 64, 896
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16).view(np.uint16)
    W.ravel()[::53] = 0x0201  # fp16 subnormals: flushed by the reference decode
    x = rng.uniform(-1, 1, K).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float16).view(np.uint16)
    y = np.zeros(N, dtype=np.float32)
    P = ctypes.c_void_p
    L.ref_gemv_h(W.ctypes.data_as(P), x.ctypes.data_as(P), b.ctypes.data_as(P), y.ctypes.data_as(P), K, N)
    return {"rng": "numpy default_rng(1): W=N(0,.02) fp16 [64x896] with every 53rd = 0x0201, "
                   "x=U(-1,1) K, bias=N(0,.02) fp16 N", "y": fhex(y),
            "source": "gpu-llm/engine/qwen_engine.c cpu_gemv_h (reference, unmodified)"}


def main():
    if not orc.ref_available():
        sys.exit("oracle/_ref is not built: make -C oracle ref REF=<reference checkout>")
    qpath = conftest._synth(sb200.MODEL_QWEN, "qwen", conftest.QWEN_SEED, sb200.QWEN["FILE_BYTES"])
    gpath = conftest._synth(sb200.MODEL_GPT2, "gpt2", conftest.GPT2_SEED, sb200.GPT2["TOTAL_FLOATS"] * 4)
    out = {
        "qwen_decode.json": engine_fixture("qwen", qpath, conftest.QWEN_SEED, sb200.QWEN["V"], 4, 101),
        "gpt2_decode.json": engine_fixture("gpt2", gpath, conftest.GPT2_SEED, sb200.GPT2["V"], 4, 102),
        "gemv_h.json": gemv_h_fixture(),
    }
    for fn, obj in out.items():
        with open(os.path.join(HERE, fn), "w") as f:
            json.dump(obj, f, indent=1)
        print("wrote", fn)


if __name__ == "__main__":
    main()
