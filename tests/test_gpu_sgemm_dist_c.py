"""The multi-GPU SGEMM from the C host: `gpu_workload --gpus N` runs the
row-panel product (sb_sgemm_rows) with an in-place NCCL all-gather of C
(sb_sgemm_panel_allgather) on each device's primary context, one host
thread per rank, and every rank checks sampled cells of every panel of its
gathered C against the harness's CPU loop (gpu_workload.c:97-101).

Failure detection without a GPU fault: a communicator whose second rank
never joins must give up at its deadline (non-blocking init, polled
ncclCommGetAsyncError, then ncclCommAbort) and return an error -- no kernel
is involved.  That check runs in a child process, so even a stuck abort
could not hang the test session."""
import json
import os
import subprocess
import sys

import pytest

import sb200

pytestmark = pytest.mark.gpu
BIN = os.path.join(os.path.dirname(sb200.__file__), "bin")


def _workload(gpus, n):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    out = subprocess.run(["timeout", "-k", "20", "600", os.path.join(BIN, "gpu_workload"), "--json", "--sizes", "256",
                          "--membw-mib", "256", "--gpus", str(gpus), "--dist-n", str(n)],
                         capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stderr[-1500:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("n", [2048, 1000])
def test_gpu_workload_dist_one_gpu(cuda_dev, n):
    """One rank: the NCCL communicator, panel product and (trivial) gather
    path of the C host; n = 1000 leaves a ragged last tile."""
    j = _workload(1, n)
    d = j["sgemm_dist"]
    assert d["gpus"] == 1 and d["n"] == n and d["verdict"] == "CORRECT" and d["cells_checked"] == 16
    assert d["compute_ms"] > 0 and d["tflops"] > 0
    assert j["kernels"]["sgemm"] == "CORRECT" and j["done"] is True


def test_gpu_workload_dist_two_gpus(cuda_dev):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    d = _workload(2, 4096)["sgemm_dist"]
    assert d["gpus"] == 2 and d["verdict"] == "CORRECT" and d["cells_checked"] == 2 * 2 * 16
    assert d["allgather_ms"] >= 0


_NEVER_JOINS = r"""
import ctypes, sys, time
sys.path.insert(0, sys.argv[1])
import sb200
sb200.init(0)
L = sb200.lib()
uid = ctypes.create_string_buffer(128)
sb200.check(L.sb_nccl_unique_id(uid))
comm = ctypes.c_void_p()
t0 = time.time()
rc = L.sb_nccl_comm_init(ctypes.byref(comm), 2, uid, 0, ctypes.c_double(3.0))  # rank 1 never calls
dt = time.time() - t0
msg = L.sb_last_error().decode()
print("RC", rc, "DT %.1f" % dt, "MSG", msg, flush=True)
# the process is still usable: a one-rank communicator works afterwards
uid2 = ctypes.create_string_buffer(128)
sb200.check(L.sb_nccl_unique_id(uid2))
c1 = ctypes.c_void_p()
sb200.check(L.sb_nccl_comm_init(ctypes.byref(c1), 1, uid2, 0, ctypes.c_double(60.0)))
sb200.check(L.sb_nccl_comm_destroy(c1, ctypes.c_double(60.0)))
print("AFTER OK", flush=True)
"""


def test_nccl_init_times_out_when_a_rank_never_joins(cuda_dev):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    out = subprocess.run(["timeout", "-k", "10", "120", sys.executable, "-c", _NEVER_JOINS,
                          os.path.dirname(sb200.__file__)], capture_output=True, text=True, env=env)
    assert out.returncode == 0, out.stdout[-800:] + out.stderr[-1500:]
    line = next(ln for ln in out.stdout.splitlines() if ln.startswith("RC"))
    parts = line.split()
    assert int(parts[1]) != 0 and "timed out" in line, line
    assert float(parts[3]) < 30.0, line
    assert "AFTER OK" in out.stdout
