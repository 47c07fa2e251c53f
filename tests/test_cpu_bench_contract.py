"""CPU check of bench.py's reference arm: `bench.py --impl reference` times
the reference's own CPU decode (oracle/_ref) and prints one JSON line with
the headline metric, unit and direction, the reference-arm markers and its
CPU baseline (a short run: one step of two tokens per host core)."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BENCH = os.path.join(REPO, "oracle", "_ref", "ref_qwen_bench")


# runs bench.py in-process, then reports whether this package's GPU library
# was ever mapped into that process
_MAPS_PROBE = """
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("MAPPED_PRODUCT_LIB" if "libswitch_b200" in maps else "NO_PRODUCT_LIB")
"""


@pytest.mark.skipif(not os.access(REF_BENCH, os.X_OK), reason="oracle/_ref not built (needs the reference sources)")
def test_reference_arm_json_line():
    """One JSON line with the headline metric; the reference arm primes the
    same 32-token prompt as the GPU arm and never maps libswitch_b200.so."""
    out = subprocess.run([sys.executable, "-c", _MAPS_PROBE], capture_output=True, text=True, timeout=900, cwd=REPO)
    assert out.returncode == 0, out.stderr[-800:]
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "NO_PRODUCT_LIB"
    line = json.loads(lines[-2])
    assert line["impl"] == "reference"
    assert line["metric"] == "Qwen-0.5B-shape FP16 decode tok/s" and line["unit"] == "tok/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["steps"] == 1 and line["warmup"] == 0
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["config"]["n_prompt"] == 32 and line["config"]["workload"].endswith("(configs[2])")
    assert "positions 32+" in cb["sample"]


def test_synth_tool_matches_library():
    """bin/sb_synth (no CUDA) writes the prompt ids the library's
    sb_synth_ids writes: both arms of the bench decode the same prompt."""
    sys.path.insert(0, os.path.join(REPO, "switch-l4t-gpu_b200"))
    import sb200
    exe = os.path.join(REPO, "switch-l4t-gpu_b200", "bin", "sb_synth")
    out = subprocess.run([exe, "ids", "32", "151936", "1000"], capture_output=True, text=True, check=True)
    assert [int(v) for v in out.stdout.split()] == sb200.synth_ids(32, 151936, 1000)
