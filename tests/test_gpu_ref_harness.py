"""The reference's own driver-API harnesses, unmodified, on the B200.

`gpu_workload.c` and `gpu-llm/harness/gemv_test.c` are compiled from the
reference's sources exactly as their headers say (`gcc ... -lcuda -lm`, the
`oracle/Makefile` targets `gpu_workload_drv` and `gemv_test_drv`), so they
bind the real driver, create their own context with cuCtxCreate_v2, load the
module image named on the command line with cuModuleLoadData and launch the
kernels by name with their stock geometry (gpu_workload.c:65-74, :93-177,
:209; gemv_test.c:65-73, :107-110).  Pointed at this package's images they
must print the reference's own verdicts: every SGEMM kernel CORRECT against
its serial loop (0.05|ref| + 1e-3, gpu_workload.c:97-101) and every GEMV
CORRECT against its golden loop (1e-4 rel + abs, gemv_test.c:118-122).

These binaries are built from the reference checkout; where they were not
built the test is skipped."""
import json
import os
import subprocess

import pytest

import orc
import sb200

pytestmark = pytest.mark.gpu
LIB = os.path.join(os.path.dirname(sb200.__file__), "lib")


def _exe(name):
    p = os.path.join(orc.REF_DIR, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not built (make -C oracle ref REF=<reference checkout>)")
    return p


def test_reference_gpu_workload_on_switch_gpu_image():
    exe = _exe("gpu_workload_drv")
    img = os.path.join(LIB, "switch_gpu.cubin")
    out = subprocess.run([exe, "--json", img], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    j = json.loads(out.stdout)
    assert j["done"] is True
    assert j["kernels"] == {"sgemm": "CORRECT", "sgemm_naive": "CORRECT",
                            "sgemm_tiled4": "CORRECT", "sgemm_opt": "CORRECT"}
    for key in ("sgemm", "sgemm4", "sgemm_opt"):
        assert [r["n"] for r in j[key]] == [256, 512, 1024]
        assert all(r["gflops"] > 0 for r in j[key])
    assert j["membw_gbps"] > 0
    # the human-readable form ends with the marker the task consumer matches
    out = subprocess.run([exe, img], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0 and out.stdout.rstrip().endswith("WORKLOAD_DONE")
    assert "sgemm 256: CORRECT" in out.stdout and "sgemm_naive 256: CORRECT (0 bad cells)" in out.stdout


@pytest.mark.parametrize("n,k", [(4096, 4096), (896, 4864), (1001, 1028)])
def test_reference_gemv_test_on_gemv_image(n, k):
    exe = _exe("gemv_test_drv")
    img = os.path.join(LIB, "gemv.cubin")
    out = subprocess.run([exe, img, str(n), str(k)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "GEMV_TEST_DONE" in out.stdout
    for name in ("gemv", "gemv4", "gemv_warp"):
        assert f"{name}: CORRECT" in out.stdout
