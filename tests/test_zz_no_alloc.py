"""The allocation-free decode attention entry point, sb_attn_decode_noalloc.

It exists for callers that cannot allocate device memory -- hosts that fix
their device budget at start-up (as the reference's Tegra engines do),
frameworks that own every allocation, token loops that must not allocate --
so its split-T scratch lives in a static array inside the library.  These
tests call it through the C-ABI and compare it with the CPU oracle's
attention (the reference's scores -> softmax -> mix, qwen_engine.c:318-331
and gpt2_engine.c:379-397) and with sb_attn_decode (the caller-scratch
entry point) under the attention tests' tolerance, on calls made back to
back with different shapes (the shared array keeps the previous call's
contents), and check that sizes beyond its limit are refused.  This file is
collected last on purpose."""
import numpy as np
import pytest

import orc
import sb200

pytestmark = pytest.mark.gpu


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _case(T, model, seed):
    if model == "qwen":
        NH, NKV, stride = 14, 2, 128
    else:
        NH, NKV, stride = 12, 12, 768
    q = sb200.synth_uniform(NH * 64, -1, 1, seed)
    kc = sb200.synth_uniform(T * stride, -1, 1, seed + 1)
    vc = sb200.synth_uniform(T * stride, -1, 1, seed + 2)
    if model == "qwen":
        ref = orc.attn_qwen(q, kc, vc, T, NH, NKV, 64, stride, 0.125)
    else:
        ref = orc.attn_gpt2(q, kc, vc, T, NH, 64, stride, 0.125)
    return NH, NKV, stride, _t(q), _t(kc), _t(vc), ref


def _with_scratch(T, NH, NKV, stride, q, kc, vc):
    import torch
    part = torch.zeros(NKV * ((T + 15) // 16) * (NH // NKV) * 66, device="cuda")
    counters = torch.zeros(NKV, dtype=torch.int32, device="cuda")
    out = torch.zeros(NH * 64, device="cuda")
    sb200.attn_decode(q, kc, vc, out, T, NH, NKV, 64, stride, 0.125, part, counters)
    return out


@pytest.mark.parametrize("T,model,seed", [(288, "qwen", 1), (37, "gpt2", 2), (2048, "qwen", 3), (1, "gpt2", 4),
                                          (1, "qwen", 6), (2048, "gpt2", 7)])
def test_noalloc_matches_oracle_and_scratch_entry_point(cuda_dev, T, model, seed):
    import torch
    NH, NKV, stride, q, kc, vc, ref = _case(T, model, seed)
    want = _with_scratch(T, NH, NKV, stride, q, kc, vc).cpu().numpy()
    got = torch.full((NH * 64,), float("nan"), device="cuda")
    sb200.attn_decode_noalloc(q, kc, vc, got, T, NH, NKV, 64, stride, 0.125)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=2e-6)


def test_noalloc_two_calls_in_a_row(cuda_dev):
    """Back-to-back calls of different shapes on the shared array, then the
    same call twice: each agrees with the oracle."""
    import torch
    for T, model, seed in ((500, "qwen", 9), (61, "gpt2", 10), (500, "qwen", 9)):
        NH, NKV, stride, q, kc, vc, ref = _case(T, model, seed)
        want = _with_scratch(T, NH, NKV, stride, q, kc, vc).cpu().numpy()
        got = torch.zeros(NH * 64, device="cuda")
        sb200.attn_decode_noalloc(q, kc, vc, got, T, NH, NKV, 64, stride, 0.125)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-5, atol=2e-6)
        np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=2e-6)


def test_noalloc_rejects_beyond_limit(cuda_dev):
    import torch
    NH, NKV, stride, q, kc, vc, _ = _case(4, "qwen", 5)
    out = torch.zeros(NH * 64, device="cuda")
    with pytest.raises(sb200.SbError, match="2048"):
        sb200.attn_decode_noalloc(q, kc, vc, out, 2049, NH, NKV, 64, stride, 0.125)
    with pytest.raises(sb200.SbError):
        sb200.attn_decode_noalloc(q, kc, vc, out, 4, 32, 32, 64, 32 * 64, 0.125)


def test_noalloc_in_a_host_created_context(cuda_dev):
    """The reference's hosts run on a context they create themselves
    (cuCtxCreate_v2, gpu_workload.c:67), not the primary one.  There the
    entry point uses that context's own copy of the static array: the result
    matches the oracle, and afterwards a call back on the primary context
    (torch's) still does."""
    import ctypes

    import torch

    import drv
    cu = drv.cuda()
    T, NH, NKV, stride = 300, 14, 2, 128
    q = sb200.synth_uniform(NH * 64, -1, 1, 31)
    kc = sb200.synth_uniform(T * stride, -1, 1, 32)
    vc = sb200.synth_uniform(T * stride, -1, 1, 33)
    ref = orc.attn_qwen(q, kc, vc, T, NH, NKV, 64, stride, 0.125)
    dev = ctypes.c_int()
    drv.check(cu.cuDeviceGet(ctypes.byref(dev), 0), "cuDeviceGet")
    ctx = ctypes.c_void_p()
    drv.check(cu.cuCtxCreate_v2(ctypes.byref(ctx), 0, dev), "cuCtxCreate_v2")
    bufs = []
    try:
        def upload(a):
            p = ctypes.c_uint64()
            drv.check(cu.cuMemAlloc_v2(ctypes.byref(p), ctypes.c_size_t(a.nbytes)), "cuMemAlloc_v2")
            bufs.append(p)
            drv.check(cu.cuMemcpyHtoD_v2(p, a.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(a.nbytes)), "HtoD")
            return p.value
        dq, dk, dv = upload(q), upload(kc), upload(vc)
        out = np.full(NH * 64, np.nan, dtype=np.float32)
        dout = upload(out)
        for _ in range(2):
            sb200.check(sb200.lib().sb_attn_decode_noalloc(ctypes.c_void_p(dq), ctypes.c_void_p(dk),
                                                           ctypes.c_void_p(dv), ctypes.c_void_p(dout), T, NH, NKV,
                                                           64, stride, ctypes.c_float(0.125), None))
            drv.check(cu.cuCtxSynchronize(), "cuCtxSynchronize")
            drv.check(cu.cuMemcpyDtoH_v2(out.ctypes.data_as(ctypes.c_void_p), ctypes.c_uint64(dout),
                                         ctypes.c_size_t(out.nbytes)), "DtoH")
            np.testing.assert_allclose(out, ref, rtol=1e-5, atol=2e-6)
    finally:
        for p in bufs:
            cu.cuMemFree_v2(p)
        drv.check(cu.cuCtxDestroy_v2(ctx), "cuCtxDestroy_v2")  # pops it: torch's context is current again
    NH, NKV, stride, q2, kc2, vc2, ref2 = _case(T, "qwen", 34)
    got = torch.zeros(NH * 64, device="cuda")
    sb200.attn_decode_noalloc(q2, kc2, vc2, got, T, NH, NKV, 64, stride, 0.125)
    torch.cuda.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), ref2, rtol=1e-5, atol=2e-6)
