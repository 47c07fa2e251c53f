"""Row-panel sharded SGEMM on GPUs: the single-rank path in process, and
2 ranks over NCCL (torch.distributed.run) when two GPUs are visible.
Bars: relative Frobenius error <= 1e-5 against the oracle's restatement of
the harness loop (gpu_workload.c:97-98) on sampled rows, and a Freivalds
check of the whole product."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import orc
import sb200
import sgemm_dist

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("M,N,K", [(1000, 384, 1002), (4096, 4096, 512)])
def test_single_rank_panel(cuda_dev, M, N, K):
    import torch
    A = sb200.synth_uniform(M * K, -1.0, 1.0, 3).reshape(M, K)
    B = sb200.synth_uniform(K * N, -1.0, 1.0, 4).reshape(K, N)
    ps = sgemm_dist.PanelSgemm(M, N, K)
    assert (ps.row0, ps.row1, ps.world) == (0, M, 1)
    C = ps(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()).cpu().numpy()
    rows = list(range(0, M, max(1, M // 32))) + [M - 1]
    want = orc.sgemm(A, B, 0, M)[rows] if M <= 1024 else np.stack([orc.sgemm(A[r:r + 1], B)[0] for r in rows])
    rel = np.linalg.norm(C[rows] - want) / np.linalg.norm(want)
    assert rel <= 1e-5
    assert orc.freivalds(A, B, np.ascontiguousarray(C)) <= 1e-5


def test_ipc_stores_from_another_process(cuda_dev):
    """The peer-store path on one GPU: this process exports C (CUDA IPC), a
    child process maps it and runs sb_sgemm_multi into its own buffer and
    into this C.  Every cell arrives, bit-identical to this process's own
    sgemm_b200 launch, within the FP32 bar of the harness loop.  (The two
    processes' kernels never wait on each other.)"""
    import torch
    import drv
    M, N, K, seed = 512, 384, 256, 77
    A = sb200.synth_uniform(M * K, -1.0, 1.0, seed).reshape(M, K)
    B = sb200.synth_uniform(K * N, -1.0, 1.0, seed + 1).reshape(K, N)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    handle, offset = sb200.ipc_export(C)
    cmd = [sys.executable, os.path.join(HERE, "ipc_sgemm_worker.py"), handle.hex(), str(offset),
           str(M), str(N), str(K), str(seed)]
    r = subprocess.run(["timeout", "-k", "10", "120"] + cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    want = torch.zeros((M, N), device="cuda")
    drv.Module(sb200.CUBINS["switch_gpu"]).launch("sgemm_b200", ((M // 128) * (N // 128),), (256,), dA, dB, want,
                                                  M, N, K)
    torch.cuda.synchronize()
    assert torch.equal(C, want)
    assert float(r.stdout.split()[-1]) == float(want.double().sum())
    ref = orc.sgemm(A, B)
    rows = [0, 255, 511]
    assert np.linalg.norm(C.cpu().numpy()[rows] - ref[rows]) <= 1e-5 * np.linalg.norm(ref[rows])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_nccl_allgather_and_peer_stores(cuda_dev):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.join(HERE, "dist_sgemm_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "400"] + cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    import dist_sgemm_worker
    assert r.stdout.count(" ok") == 2 * len(dist_sgemm_worker.CASES), r.stdout
