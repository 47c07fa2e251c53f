"""Opt-in 3xTF32 tensor-core SGEMM against the oracle's restatement of the
harness loop (gpu_workload.c:97-98): the FP32 bar, relative Frobenius error
<= 1e-5, plus a Freivalds check of whole products; edge tiles (M, N not
multiples of 128, K not a multiple of 32) and split-K launches (fewer tiles
than SMs) included."""
import numpy as np
import pytest

import orc
import sb200
import sgemm_dist

pytestmark = pytest.mark.gpu
REL_FROB = 1e-5


def _mats(M, N, K, seed):
    A = sb200.synth_uniform(M * K, -1.0, 1.0, seed).reshape(M, K)
    B = sb200.synth_uniform(K * N, -1.0, 1.0, seed + 1).reshape(K, N)
    return A, B


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (1000, 384, 1004), (257, 132, 68), (128, 128, 32),
                                   # prompt-prefill shapes: fewer tiles than SMs, K split over CTAs
                                   (15, 2304, 768), (15, 768, 3072), (140, 3072, 768), (1, 768, 768)])
def test_3xtf32_matches_oracle(cuda_dev, M, N, K):
    import torch
    A, B = _mats(M, N, K, 40 + M)
    dC = torch.full((M, N), float("nan"), device="cuda")
    sb200.sgemm_3xtf32(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC, M, N, K)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    C = dC.cpu().numpy()
    assert np.isfinite(C).all()
    ref = orc.sgemm(A, B)
    rel = np.linalg.norm((C - ref).astype(np.float64)) / np.linalg.norm(ref.astype(np.float64))
    assert rel <= REL_FROB, f"rel {rel:.2e}"
    assert orc.sgemm_bad_cells(C, ref) == 0


def test_3xtf32_large_freivalds(cuda_dev):
    import torch
    M = N = 4096
    K = 2048
    A, B = _mats(M, N, K, 77)
    dC = torch.empty(M, N, device="cuda")
    sb200.sgemm_3xtf32(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC, M, N, K)
    C = dC.cpu().numpy()
    assert sb200.tc_error() == 0
    assert orc.freivalds(A, B, C) <= REL_FROB
    rows = [0, 1, 1000, 4095]
    want = np.stack([orc.sgemm(A[r:r + 1], B)[0] for r in rows])
    assert np.linalg.norm(C[rows] - want) / np.linalg.norm(want) <= REL_FROB


def test_3xtf32_panel_path(cuda_dev):
    import torch
    M, N, K = 1000, 512, 256
    A, B = _mats(M, N, K, 9)
    ps = sgemm_dist.PanelSgemm(M, N, K, kernel="3xtf32")
    C = ps(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()).cpu().numpy()
    ref = orc.sgemm(A, B)
    assert np.linalg.norm(C - ref) / np.linalg.norm(ref) <= REL_FROB


def test_3xtf32_rejects_unaligned_shapes(cuda_dev):
    import torch
    A = torch.zeros(8, 6, device="cuda")
    B = torch.zeros(6, 8, device="cuda")
    C = torch.zeros(8, 8, device="cuda")
    with pytest.raises(sb200.SbError):
        sb200.sgemm_3xtf32(A, B, C, 8, 8, 6)  # K % 4 != 0


def test_3xtf32_16384_accuracy(cuda_dev):
    """The bench size: Freivalds check of the whole 16384^3 product."""
    import torch
    n = 16384
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    A = torch.rand(n, n, generator=g, device="cuda") * 2 - 1
    B = torch.rand(n, n, generator=g, device="cuda") * 2 - 1
    C = torch.empty(n, n, device="cuda")
    sb200.sgemm_3xtf32(A, B, C, n, n, n)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    rel = orc.freivalds(A.cpu().numpy(), B.cpu().numpy(), C.cpu().numpy())
    assert rel <= REL_FROB, f"freivalds {rel:.2e}"


@pytest.mark.parametrize("M,N,K,nout", [(2048, 2048, 512, 2), (256, 384, 64, 3)])
def test_3xtf32_multi_outputs(cuda_dev, M, N, K, nout):
    """sb_sgemm_3xtf32_multi stores every row of every tile into each output
    (here all on this GPU): every output within the FP32 bar of the harness
    loop, all outputs identical, and bit-identical to sb_sgemm_3xtf32 when
    that call needs no K split (tiles >= SMs)."""
    import torch
    A = sb200.synth_uniform(M * K, -1.0, 1.0, 61).reshape(M, K)
    B = sb200.synth_uniform(K * N, -1.0, 1.0, 62).reshape(K, N)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    outs = [torch.full((M, N), float("nan"), device="cuda") for _ in range(nout)]
    sb200.sgemm_3xtf32_multi(dA, dB, outs, M, N, K)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    if (M // 128) * (N // 128) >= sb200.sm_count():
        one = torch.zeros((M, N), device="cuda")
        sb200.sgemm_3xtf32(dA, dB, one, M, N, K)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], one)
    C = outs[0].cpu().numpy()
    rows = sorted({0, M // 2, M - 1})
    ref = np.stack([orc.sgemm(A, B, r, r + 1)[r] for r in rows])
    assert np.linalg.norm(C[rows] - ref) <= 1e-5 * np.linalg.norm(ref)
