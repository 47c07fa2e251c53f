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
