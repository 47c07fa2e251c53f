"""GEMV parity on the GPU against the oracle (cpu_gemv_h qwen_engine.c:276-284,
cpu_gemv gpt2_engine.c:342-349, gemv_test.c:85-90).

Tolerance: |y - ref| <= 1e-4 |ref| + 1e-4, the reference GEMV harness's own
rule (gemv_test.c:119).  Shapes are every decode-step matrix of both models
plus ragged ones (N % 8 != 0, K % 8 == 4, N = 50257, 151936)."""
import numpy as np
import pytest

import drv
import orc
import sb200

pytestmark = pytest.mark.gpu


def _close(y, ref):
    bad = np.abs(y - ref) > 1e-4 * np.abs(ref) + 1e-4
    assert np.isfinite(y).all()
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; max err {np.abs(y - ref).max():.3e}"


def _wh(N, K, seed):
    W = sb200.synth_normal_h(N * K, 0.02, seed).reshape(N, K)
    # plant fp16 subnormals / zeros so the flush-to-zero decode is exercised
    W.ravel()[::97] = 0x0003
    W.ravel()[1::101] = 0x8201
    return W


def _x(K, seed):
    return sb200.synth_uniform(K, -1.0, 1.0, seed)


@pytest.fixture(scope="module")
def qmod(cuda_dev):
    return drv.Module(sb200.CUBINS["qwen"])


@pytest.fixture(scope="module")
def gmod(cuda_dev):
    return drv.Module(sb200.CUBINS["gpt2"])


@pytest.fixture(scope="module")
def m0mod(cuda_dev):
    return drv.Module(sb200.CUBINS["gemv"])


QWEN_SHAPES = [(1152, 896, True), (896, 896, False), (9728, 896, False), (896, 4864, False),
               (151936, 896, False), (1001, 896, True), (7, 64, False)]


@pytest.mark.parametrize("N,K,bias", QWEN_SHAPES)
def test_gemv_h_dropin(cuda_dev, qmod, N, K, bias):
    import torch
    W = _wh(N, K, N + K)
    x = _x(K, 1)
    b = sb200.synth_uniform(N, -0.05, 0.05, 2) if bias else None
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dx = torch.from_numpy(x).cuda()
    db = torch.from_numpy(b).cuda() if bias else None
    dy = torch.full((N,), float("nan"), device="cuda")
    qmod.launch("gemv_h", ((N + 7) // 8,), (256,), dW, dx, db, dy, K, N)  # qwen_engine.c:219
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), orc.gemv_h(W, x, b))


@pytest.mark.parametrize("N,K,bias", QWEN_SHAPES)
def test_gemv_h_abi(cuda_dev, N, K, bias):
    import torch
    W = _wh(N, K, 3 * N + K)
    x = _x(K, 4)
    b = sb200.synth_uniform(N, -0.05, 0.05, 5) if bias else None
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dx = torch.from_numpy(x).cuda()
    db = torch.from_numpy(b).cuda() if bias else None
    dy = torch.full((N,), float("nan"), device="cuda")
    sb200.gemv_h(dW, dx, db, dy, K, N)
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), orc.gemv_h(W, x, b))


def test_gemv_h_dropin_k_mod8_is_4(cuda_dev, qmod):
    """The reference only requires K % 4 == 0 (qwen_kernels.cu:32)."""
    import torch
    N, K = 100, 44
    W = _wh(N, K, 8)
    x = _x(K, 9)
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = torch.zeros(N, device="cuda")
    qmod.launch("gemv_h", ((N + 7) // 8,), (256,), dW, dx, None, dy, K, N)
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), orc.gemv_h(W, x))


@pytest.mark.parametrize("B", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("N,K", [(896, 896), (4864, 896), (896, 4864), (1003, 8192), (3, 8), (7, 13696),
                                 (1180, 1024), (1184, 1024)])
def test_gemv_hh_batched(cuda_dev, B, N, K):
    """FP16 activations (the GEMV sweep's x), batch B: y_b = W h2f(x_b).
    Fewer than 2 x SMs four-row tasks (N < 1184 on 148 SMs) take the split-K
    kernels, the rest the warp-per-task ones; both sides of the switch, ragged
    row tails and K slices shorter than a warp's stride are covered."""
    import torch
    W = _wh(N, K, 17)
    X = sb200.synth_normal_h(B * K, 1.0, 18).reshape(B, K)
    dW = torch.from_numpy(W.view(np.int16)).cuda()
    dX = torch.from_numpy(X.view(np.int16)).cuda()
    dY = torch.full((B, N), float("nan"), device="cuda")
    sb200.gemv_hh(dW, dX, dY, K, N, B)
    torch.cuda.synchronize()
    Y = dY.cpu().numpy()
    for b in range(B):
        _close(Y[b], orc.gemv_h(W, orc.h2f(X[b])))


@pytest.mark.parametrize("name,grid_div", [("gemv", 256), ("gemv4", 256), ("gemv_warp", 8)])
def test_m0_gemv_stock(cuda_dev, m0mod, name, grid_div):
    """gemv_test.c defaults: 4096x4096 FP32, launch grid per gemv_test.c:109."""
    import torch
    N = K = 4096
    W = sb200.synth_uniform(N * K, -0.5, 0.5, 42).reshape(N, K)
    x = sb200.synth_uniform(K, -0.5, 0.5, 43)
    dW, dx = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    dy = torch.zeros(N, device="cuda")
    m0mod.launch(name, ((N + grid_div - 1) // grid_div,), (256,), dW, dx, dy, K, N)
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), orc.gemv_f32(W, x))


GPT2_SHAPES = [(2304, 768), (768, 768), (3072, 768), (768, 3072), (50257, 768), (13, 12)]


@pytest.mark.parametrize("N,K", GPT2_SHAPES)
@pytest.mark.parametrize("bias", [False, True])
def test_gpt2_gemv_dropins(cuda_dev, gmod, N, K, bias):
    import torch
    W = sb200.synth_uniform(N * K, -0.05, 0.05, N).reshape(N, K)
    x = _x(K, 6)
    b = sb200.synth_uniform(N, -0.05, 0.05, 7) if bias else None
    dW, dx = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    dy = torch.zeros(N, device="cuda")
    if bias:
        gmod.launch("gemv_warp_b", ((N + 7) // 8,), (256,), dW, dx, torch.from_numpy(b).cuda(), dy, K, N)
    else:
        gmod.launch("gemv_warp", ((N + 7) // 8,), (256,), dW, dx, dy, K, N)
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), orc.gemv_f32(W, x, b))
    # the tuned C-ABI path too
    dy2 = torch.zeros(N, device="cuda")
    sb200.gemv_f32(dW, dx, torch.from_numpy(b).cuda() if bias else None, dy2, K, N)
    torch.cuda.synchronize()
    _close(dy2.cpu().numpy(), orc.gemv_f32(W, x, b))


@pytest.mark.parametrize("T", [1, 16, 17, 40])
def test_gemv_multi_stock(cuda_dev, gmod, T):
    """gemv_multi at the QKV shape, grid (ceil(N/8), ceil(T/16)) as
    gpt2_engine.c:280."""
    import torch
    N, K = 2304, 768
    W = sb200.synth_uniform(N * K, -0.05, 0.05, 21).reshape(N, K)
    X = sb200.synth_uniform(T * K, -1, 1, 22).reshape(T, K)
    b = sb200.synth_uniform(N, -0.05, 0.05, 23)
    dW, dX, db = torch.from_numpy(W).cuda(), torch.from_numpy(X).cuda(), torch.from_numpy(b).cuda()
    dY = torch.zeros((T, N), device="cuda")
    gmod.launch("gemv_multi", ((N + 7) // 8, (T + 15) // 16), (256,), dW, dX, db, dY, K, N, T)
    torch.cuda.synchronize()
    ref = orc.gemv_multi_f32(W, X, b)
    _close(dY.cpu().numpy().ravel(), ref.ravel())
