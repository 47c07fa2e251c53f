"""Tensor-core (tcgen05) batched FP16 GEMM against the oracle's restatement
of the reference fp16 GEMV (cpu_gemv_h, qwen_engine.c:276-284) applied to
each activation row.  Inputs have fp16 subnormals flushed, so the tensor
pipe (which keeps subnormals) and the reference decode (which zeroes them)
read the same values.  Bar: relative Frobenius error <= 1e-4 per batch
(FP32 accumulation on the tensor pipe, K up to 8192)."""
import numpy as np
import pytest

import orc
import sb200

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _flushed_h(n, std, seed):
    h = sb200.synth_normal_h(n, std, seed)
    h[(h & 0x7C00) == 0] = 0
    return h


@pytest.mark.parametrize("N,K", [(896, 896), (4864, 896), (896, 4864), (1000, 264), (130, 72), (151936, 896)])
@pytest.mark.parametrize("B", [1, 4, 16, 24])
def test_gemm_hh_matches_oracle(cuda_dev, N, K, B):
    import torch
    if N == 151936 and B not in (1, 16):
        pytest.skip("large shape: two batch widths suffice")
    W = _flushed_h(N * K, 0.02, 11 + K).reshape(N, K)
    X = _flushed_h(B * K, 1.0, 17 + N).reshape(B, K)
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dX = torch.from_numpy(X.view(np.int16)).cuda()
    dY = torch.full((B, N), float("nan"), device="cuda")
    sb200.gemm_hh(dW, dX, dY, K, N, B)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    Y = dY.cpu().numpy()
    assert np.isfinite(Y).all()
    rows = range(B) if N * K <= 8 << 20 else [0, B - 1]
    for b in rows:
        want = orc.gemv_h(W, orc.h2f(X[b]))
        rel = np.linalg.norm((Y[b] - want).astype(np.float64)) / np.linalg.norm(want.astype(np.float64))
        assert rel <= TOL, f"batch row {b}: rel {rel:.2e}"


def test_gemm_hh_matches_cuda_core_gemv(cuda_dev):
    """Same inputs through gemv_hh (CUDA cores, batch <= 8): the two agree."""
    import torch
    N, K, B = 4864, 896, 8
    W = _flushed_h(N * K, 0.02, 5).reshape(N, K)
    X = _flushed_h(B * K, 1.0, 6).reshape(B, K)
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dX = torch.from_numpy(X.view(np.int16)).cuda()
    y1 = torch.empty(B, N, device="cuda")
    y2 = torch.empty(B, N, device="cuda")
    sb200.gemm_hh(dW, dX, y1, K, N, B)
    sb200.gemv_hh(dW, dX, y2, K, N, B)
    torch.cuda.synchronize()
    a, b = y1.cpu().numpy().astype(np.float64), y2.cpu().numpy().astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) <= TOL


def test_gemm_hh_rejects_bad_shapes(cuda_dev):
    import torch
    W = torch.zeros(64, 12, dtype=torch.int16, device="cuda")
    X = torch.zeros(2, 12, dtype=torch.int16, device="cuda")
    Y = torch.zeros(2, 64, device="cuda")
    with pytest.raises(sb200.SbError):
        sb200.gemm_hh(W, X, Y, 12, 64, 2)  # K % 8 != 0
    with pytest.raises(sb200.SbError):
        sb200.gemm_hh(W, X, Y, 8, 64, 257)  # batch > 256


# (batches of 16 rows or fewer on shorter outputs run on mma.sync tiles, not
# on this kernel: both cases keep B > 16)
@pytest.mark.parametrize("N,K,B,skip", [(1024, 1024, 32, 0), (4096, 2048, 24, 5)])
def test_gemm_hh_wait_timeout_recovers(cuda_dev, N, K, B, skip):
    """Failure detection on the tensor-core kernel without a GPU fault: the
    test hook makes every TMA producer stop before K-chunk `skip`, so the
    MMA issuer's bounded wait for that stage runs out (~2 s).  The kernel
    drains the copies it issued, frees its tensor memory and returns;
    sb_tc_error reports the timeout; with the hook off the next call on the
    same context matches the oracle again."""
    import time

    import torch
    W = _flushed_h(N * K, 0.02, 5 + N).reshape(N, K)
    X = _flushed_h(B * K, 1.0, 6 + K).reshape(B, K)
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dX = torch.from_numpy(X.view(np.int16)).cuda()
    dY = torch.zeros((B, N), device="cuda")
    assert sb200.tc_error() == 0
    sb200.check(sb200.lib().sb_tc_set_test_skip(skip))
    try:
        t0 = time.time()
        sb200.gemm_hh(dW, dX, dY, K, N, B)
        torch.cuda.synchronize()
        assert sb200.tc_error() != 0
        assert time.time() - t0 < 30
    finally:
        sb200.check(sb200.lib().sb_tc_set_test_skip(-1))
    dY.fill_(float("nan"))
    sb200.gemm_hh(dW, dX, dY, K, N, B)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    Y = dY.cpu().numpy()
    for b in (0, B - 1):
        want = orc.gemv_h(W, orc.h2f(X[b]))
        rel = np.linalg.norm((Y[b] - want).astype(np.float64)) / np.linalg.norm(want.astype(np.float64))
        assert rel <= TOL


@pytest.mark.parametrize("N,K,B", [(896, 896, 4), (896, 4864, 16), (896, 896, 13), (640, 512, 24)])
def test_gemm_hh_keeps_subnormals(cuda_dev, N, K, B):
    """sb_gemm_hh uses fp16 subnormals as subnormals on both of its paths:
    small batches on short outputs (the CUDA-core form) and the tensor cores
    (B = 24).  Activation rows like the prefill's lo rows (x - fp16(x)), half
    of them subnormal, against an FP64 product of the IEEE decodes; and the
    result differs from what a flush to zero would give."""
    import torch
    rng = np.random.default_rng(N + K + B)
    W = _flushed_h(N * K, 0.02, 3 + N).reshape(N, K)
    xs = rng.normal(0, 1, (B, K)).astype(np.float32)
    hi = xs.astype(np.float16)
    lo = (xs - hi.astype(np.float32)).astype(np.float16)
    lo[:, ::2] = (lo[:, ::2].astype(np.float32) * 2.0 ** -8).astype(np.float16)  # more subnormals
    bits = lo.view(np.uint16)
    assert (((bits & 0x7C00) == 0) & ((bits & 0x3FF) != 0)).mean() > 0.3
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dX = torch.from_numpy(lo.view(np.int16).copy()).cuda()
    dY = torch.full((B, N), float("nan"), device="cuda")
    sb200.gemm_hh(dW, dX, dY, K, N, B)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    Y = dY.cpu().numpy().astype(np.float64)
    want = lo.astype(np.float64) @ W.view(np.float16).astype(np.float64).T
    rel = np.linalg.norm(Y - want) / np.linalg.norm(want)
    assert rel <= 1e-5, rel
    flushed = lo.copy()
    flushed[(flushed.view(np.uint16) & 0x7C00) == 0] = 0
    want_ftz = flushed.astype(np.float64) @ W.view(np.float16).astype(np.float64).T
    assert np.linalg.norm(Y - want_ftz) / np.linalg.norm(want_ftz) > 10 * rel
