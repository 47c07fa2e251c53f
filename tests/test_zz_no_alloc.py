"""The allocation-free decode attention entry point, sb_attn_decode_noalloc.

It exists for callers that cannot allocate device memory -- hosts that fix
their device budget at start-up (as the reference's Tegra engines do),
frameworks that own every allocation, token loops that must not allocate --
so its split-T scratch lives in a static array inside the library.  These
tests call it through the C-ABI and compare it with sb_attn_decode (the
caller-scratch entry point) under the attention tests' tolerance, on calls
made back to back with different shapes (the shared array keeps the
previous call's contents), and check that sizes beyond its limit are
refused.  This file is collected last on purpose."""
import numpy as np
import pytest

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
    return NH, NKV, stride, _t(q), _t(kc), _t(vc)


def _with_scratch(T, NH, NKV, stride, q, kc, vc):
    import torch
    part = torch.zeros(NKV * ((T + 15) // 16) * (NH // NKV) * 66, device="cuda")
    counters = torch.zeros(NKV, dtype=torch.int32, device="cuda")
    out = torch.zeros(NH * 64, device="cuda")
    sb200.attn_decode(q, kc, vc, out, T, NH, NKV, 64, stride, 0.125, part, counters)
    return out


def test_noalloc_matches_scratch_entry_point(cuda_dev):
    import torch
    for T, model, seed in ((288, "qwen", 1), (37, "gpt2", 2), (288, "qwen", 1), (2048, "qwen", 3), (1, "gpt2", 4)):
        NH, NKV, stride, q, kc, vc = _case(T, model, seed)
        want = _with_scratch(T, NH, NKV, stride, q, kc, vc)
        got = torch.full((NH * 64,), float("nan"), device="cuda")
        sb200.attn_decode_noalloc(q, kc, vc, got, T, NH, NKV, 64, stride, 0.125)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=2e-6)


def test_noalloc_two_calls_in_a_row(cuda_dev):
    import torch
    NH, NKV, stride, q, kc, vc = _case(500, "qwen", 9)
    want = _with_scratch(500, NH, NKV, stride, q, kc, vc).cpu().numpy()
    for _ in range(2):
        got = torch.zeros(NH * 64, device="cuda")
        sb200.attn_decode_noalloc(q, kc, vc, got, 500, NH, NKV, 64, stride, 0.125)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=2e-6)


def test_noalloc_rejects_beyond_limit(cuda_dev):
    import torch
    NH, NKV, stride, q, kc, vc = _case(4, "qwen", 5)
    out = torch.zeros(NH * 64, device="cuda")
    with pytest.raises(sb200.SbError, match="2048"):
        sb200.attn_decode_noalloc(q, kc, vc, out, 2049, NH, NKV, 64, stride, 0.125)
    with pytest.raises(sb200.SbError):
        sb200.attn_decode_noalloc(q, kc, vc, out, 4, 32, 32, 64, 32 * 64, 0.125)
