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


@pytest.mark.skipif(not os.access(REF_BENCH, os.X_OK), reason="oracle/_ref not built (needs the reference sources)")
def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-800:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "Qwen-0.5B-shape FP16 decode tok/s" and line["unit"] == "tok/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["steps"] == 1 and line["warmup"] == 0
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"]
