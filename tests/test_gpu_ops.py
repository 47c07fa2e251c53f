"""Decode-step building blocks on the GPU vs the oracle: norms, RoPE (bit
exact: the kernel rounds like the reference C), SwiGLU, GELU and the split-T
decode attention (GQA 14/2 and MHA 12/12) over ragged T, plus the
reference-signature attention drop-ins under their stock launches."""
import numpy as np
import pytest

import drv
import orc
import sb200

pytestmark = pytest.mark.gpu


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def qmod(cuda_dev):
    return drv.Module(sb200.CUBINS["qwen"])


@pytest.fixture(scope="module")
def gmod(cuda_dev):
    return drv.Module(sb200.CUBINS["gpt2"])


def test_rmsnorm_rows(cuda_dev):
    import torch
    n, rows = 896, 5
    x = sb200.synth_uniform(n * rows, -3, 3, 1).reshape(rows, n)
    w = sb200.synth_normal_h(n, 1.0, 2)
    y = torch.zeros((rows, n), device="cuda")
    sb200.rmsnorm(_t(x), _t(w.view(np.int16)), y, n, 1e-6, rows)
    torch.cuda.synchronize()
    for r in range(rows):
        np.testing.assert_allclose(y[r].cpu().numpy(), orc.rmsnorm(x[r], w, 1e-6), rtol=2e-6, atol=1e-7)


def test_layernorm_rows(cuda_dev):
    import torch
    n, rows = 768, 4
    x = sb200.synth_uniform(n * rows, -2, 5, 3).reshape(rows, n)
    w = sb200.synth_uniform(n, 0.5, 1.5, 4)
    b = sb200.synth_uniform(n, -0.1, 0.1, 5)
    y = torch.zeros((rows, n), device="cuda")
    sb200.layernorm(_t(x), _t(w), _t(b), y, n, 1e-5, rows)
    torch.cuda.synchronize()
    for r in range(rows):
        np.testing.assert_allclose(y[r].cpu().numpy(), orc.layernorm(x[r], w, b, 1e-5), rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("T,H,pos0", [(1, 14, 0), (1, 2, 287), (3, 14, 100), (2, 2, 8190)])
def test_rope_bit_exact(cuda_dev, T, H, pos0):
    import torch
    HD = 64
    x = sb200.synth_uniform(T * H * HD, -2, 2, 6)
    ang = np.outer(np.arange(8192, dtype=np.float64), 1e6 ** (-2.0 * np.arange(32) / 64))
    cosT, sinT = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    dx = _t(x)
    sb200.rope(dx, _t(cosT), _t(sinT), T, H, HD, pos0)
    torch.cuda.synchronize()
    assert np.array_equal(dx.cpu().numpy(), orc.rope(x, cosT, sinT, T, H, HD, pos0))


def test_swiglu_gelu(cuda_dev):
    import torch
    n = 4864
    g = sb200.synth_uniform(n, -8, 8, 7)
    u = sb200.synth_uniform(n, -2, 2, 8)
    y = torch.zeros(n, device="cuda")
    sb200.swiglu(_t(g), _t(u), y, n)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), orc.swiglu(g, u), rtol=2e-6, atol=1e-7)
    x = sb200.synth_uniform(3072, -6, 6, 9)
    z = torch.zeros(3072, device="cuda")
    sb200.gelu(_t(x), z, 3072)
    torch.cuda.synchronize()
    np.testing.assert_allclose(z.cpu().numpy(), orc.gelu(x), rtol=2e-6, atol=1e-6)  # tanhf ulps near 0


@pytest.mark.parametrize("T", [1, 2, 15, 16, 17, 33, 288, 1000, 2048])
@pytest.mark.parametrize("model", ["qwen", "gpt2"])
def test_attn_decode(cuda_dev, T, model):
    import torch
    if model == "qwen":
        NH, NKV, HD, stride, scale = 14, 2, 64, 128, 0.125
    else:
        NH, NKV, HD, stride, scale = 12, 12, 64, 768, 0.125
    q = sb200.synth_uniform(NH * HD, -1, 1, T)
    kc = sb200.synth_uniform(T * stride, -1, 1, T + 1).reshape(T, stride)
    vc = sb200.synth_uniform(T * stride, -1, 1, T + 2).reshape(T, stride)
    if model == "qwen":
        ref = orc.attn_qwen(q, kc, vc, T, NH, NKV, HD, stride, scale)
    else:
        ref = orc.attn_gpt2(q, kc, vc, T, NH, HD, stride, scale)
    part = torch.zeros(NKV * ((T + 15) // 16) * (NH // NKV) * 66, device="cuda")
    counters = torch.zeros(NKV, dtype=torch.int32, device="cuda")
    out = torch.full((NH * HD,), float("nan"), device="cuda")
    for rep in range(2):  # counters must be left zeroed for the next call
        sb200.attn_decode(_t(q), _t(kc), _t(vc), out, T, NH, NKV, HD, stride, scale, part, counters)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=2e-6)
        assert int(counters.abs().sum()) == 0


def test_attn_dropins_qwen_stock(cuda_dev, qmod):
    """attn_scores_gqa -> attn_softmax -> attn_mix_gqa with the launches of
    qwen_engine.c:231-236 reproduce the oracle's attention."""
    import torch
    T, NH, NKV, HD, KV = 37, 14, 2, 64, 128
    q = sb200.synth_uniform(NH * HD, -1, 1, 1)
    kc = sb200.synth_uniform(T * KV, -1, 1, 2)
    vc = sb200.synth_uniform(T * KV, -1, 1, 3)
    sc = torch.zeros(T * NH, device="cuda")
    pr = torch.zeros(T * NH, device="cuda")
    out = torch.zeros(NH * HD, device="cuda")
    qmod.launch("attn_scores_gqa", ((T * NH + 255) // 256,), (256,), _t(q), _t(kc), sc, T, 0.125, NH, KV, HD)
    qmod.launch("attn_softmax", (1,), (NH,), sc, pr, T, NH)
    qmod.launch("attn_mix_gqa", ((NH * HD + 255) // 256,), (256,), pr, _t(vc), out, T, NH, KV, HD)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), orc.attn_qwen(q, kc, vc, T, NH, NKV, HD, KV, 0.125),
                               rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(pr.view(T, NH).sum(0).cpu().numpy(), np.ones(NH), rtol=1e-5)


def test_attn_dropins_gpt2_stock(cuda_dev, gmod):
    """attn_scores -> attn_softmax -> attn_mix with gpt2_engine.c:199-204."""
    import torch
    T = 21
    q = sb200.synth_uniform(768, -1, 1, 4)
    kc = sb200.synth_uniform(T * 768, -1, 1, 5)
    vc = sb200.synth_uniform(T * 768, -1, 1, 6)
    sc = torch.zeros(T * 12, device="cuda")
    pr = torch.zeros(T * 12, device="cuda")
    out = torch.zeros(768, device="cuda")
    gmod.launch("attn_scores", ((T * 12 + 255) // 256,), (256,), _t(q), _t(kc), sc, T, 0.125)
    gmod.launch("attn_softmax", (1,), (12,), sc, pr, T)
    gmod.launch("attn_mix", (3,), (256,), pr, _t(vc), out, T)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), orc.attn_gpt2(q, kc, vc, T, 12, 64, 768, 0.125),
                               rtol=1e-5, atol=2e-6)


def test_qwen_elementwise_dropins(cuda_dev, qmod):
    """rmsnorm / swiglu / add2 under their stock launches."""
    import torch
    n = 896
    x = sb200.synth_uniform(n, -3, 3, 10)
    w = sb200.synth_normal_h(n, 1.0, 11)
    y = torch.zeros(n, device="cuda")
    qmod.launch("rmsnorm", (1,), (256,), _t(x), _t(w.view(np.int16)), y, n, 1e-6)
    a = torch.zeros(n, device="cuda")
    qmod.launch("add2", ((n + 255) // 256,), (256,), _t(x), _t(x), a, n)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), orc.rmsnorm(x, w, 1e-6), rtol=2e-6, atol=1e-7)
    assert np.array_equal(a.cpu().numpy(), x + x)


def test_gpt2_elementwise_dropins(cuda_dev, gmod):
    """GPT-2's add_bias and add2 (gpt2_kernels.cu:209-217, both required by
    gpt2_engine.c:124-125) under the stock launches: add2 as the residual
    adds of gpt2_engine.c:220,249 (grid 3 x 256 over C = 768), add_bias over
    the fc width, and a ragged n that leaves the last block partly idle."""
    import torch
    for n, grid in ((768, 3), (3072, 12), (1000, 4)):
        a = sb200.synth_uniform(n, -2, 2, 20 + n)
        b = sb200.synth_uniform(n, -2, 2, 21 + n)
        out = torch.full((n + 64,), 7.0, device="cuda")  # the tail past n must stay untouched
        gmod.launch("add2", (grid,), (256,), _t(a), _t(b), out, n)
        y = torch.from_numpy(np.concatenate([a, np.full(64, 5.0, np.float32)])).cuda()
        gmod.launch("add_bias", (grid,), (256,), y, _t(b), n)
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        assert np.array_equal(o[:n], a + b) and np.all(o[n:] == 7.0)
        yy = y.cpu().numpy()
        assert np.array_equal(yy[:n], a + b) and np.all(yy[n:] == 5.0)
