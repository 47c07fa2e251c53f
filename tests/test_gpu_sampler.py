"""The device half of the Qwen sampler (sb_topk_penalized) and its engine
form (sb_engine_sample) against the host sampler.

The reference's sample_token (gpu-llm/engine/qwen_engine.c:375-399)
penalises each context id once per occurrence, divides every logit by the
temperature, and takes 20 passes of first-index argmax; the device kernels
must return exactly those 20 ids and values (IEEE division and
multiplication in the same order: bit-identical).  The draw over them
(softmax, top-p, xorshift) stays on the host, so with the same state the
engine path draws the same token as sb_sample_token on the full logits --
which tests/test_cpu_sampler.py pins to the reference's own code."""
import ctypes

import numpy as np
import pytest

import sb200

pytestmark = pytest.mark.gpu
V = 151936


def _host_topk(w, ctx, k, temp=0.7, rep=1.1):
    """Steps 1-3 of sample_token restated in float32 (test oracle; pinned to
    the reference's sample_token in tests/test_cpu_sampler.py)."""
    w = w.astype(np.float32).copy()
    for t in ctx:
        if 0 <= t < len(w):
            w[t] = np.float32(w[t] / np.float32(rep)) if w[t] > 0 else np.float32(w[t] * np.float32(rep))
    w = (w / np.float32(temp)).astype(np.float32)
    idx, val = [], []
    for _ in range(k):
        b = int(np.argmax(w))  # first index of the maximum
        idx.append(b)
        val.append(w[b])
        w[b] = np.float32(-1e30)
    return np.array(idx, np.int32), np.array(val, np.float32)


def _logits(rng, ctx, n=V):
    w = rng.normal(0.0, 1.5, n).astype(np.float32)
    lead = rng.integers(0, n, 12)
    w[lead] = rng.uniform(6.0, 9.0, 12).astype(np.float32)
    if ctx:
        rep = rng.choice(ctx, size=min(4, len(ctx)), replace=False)
        w[rep] = rng.uniform(6.0, 9.5, len(rep)).astype(np.float32)
        w[rep[0]] = -w[rep[0]]
    w[lead[1]] = w[lead[0]]  # an exact tie among the leaders
    w[lead[2]] = w[lead[0]]
    return w


@pytest.mark.parametrize("n,k,nctx", [(V, 20, 300), (V, 1, 0), (V, 64, 2048), (1000, 20, 50), (1025, 20, 3),
                                      (24, 20, 40), (10, 20, 5)])
def test_topk_matches_host_steps(cuda_dev, n, k, nctx):
    import torch
    rng = np.random.default_rng(n + k + nctx)
    ctx = [int(t) for t in rng.integers(0, n, nctx)]
    if nctx >= 4:  # ids repeated several times: penalised once per occurrence
        ctx += [ctx[0]] * 3 + [ctx[1]] * 2
    w = _logits(rng, ctx, n)
    want_i, want_v = _host_topk(w, ctx, k)
    dW = torch.from_numpy(w).cuda()
    dC = torch.tensor(ctx if ctx else [0], dtype=torch.int32, device="cuda")
    di = torch.full((k,), -7, dtype=torch.int32, device="cuda")
    dv = torch.zeros(k, device="cuda")
    sb200.topk_penalized(dW, n, dC, len(ctx), 0.7, 1.1, k, di, dv)
    torch.cuda.synchronize()
    got_i, got_v = di.cpu().numpy(), dv.cpu().numpy()
    kk = min(k, n)
    assert np.array_equal(got_i[:kk], want_i[:kk])
    assert np.array_equal(got_v[:kk].view(np.uint32), want_v[:kk].view(np.uint32))
    if n < k:  # fewer ids than k: the rest are empty
        assert np.all(got_i[n:] == -1)


def test_device_candidates_draw_like_host_sampler_256(cuda_dev):
    """256 consecutive draws, context growing with the drawn ids: device
    top-20 + host draw against sb_sample_token on the full logits."""
    import torch
    L = sb200.lib()
    rng = np.random.default_rng(7)
    ctx = [int(t) for t in sb200.synth_ids(32, V, 1000)]
    s_dev, s_host = ctypes.c_uint32(1234), ctypes.c_uint32(1234)
    scratch = np.zeros(V, dtype=np.float32)
    di = torch.empty(20, dtype=torch.int32, device="cuda")
    dv = torch.empty(20, device="cuda")
    for step in range(256):
        w = _logits(rng, ctx)
        c = np.asarray(ctx, dtype=np.int32)
        want = L.sb_sample_token(w.ctypes.data, V, c.ctypes.data, len(ctx), 0.7, 20, 0.8, 1.1, ctypes.byref(s_host),
                                 scratch.ctypes.data)
        sb200.topk_penalized(torch.from_numpy(w).cuda(), V, torch.from_numpy(c).cuda(), len(ctx), 0.7, 1.1, 20, di,
                             dv)
        torch.cuda.synchronize()
        got = sb200.sample_topk(di.cpu().numpy(), dv.cpu().numpy(), 0.8, s_dev)
        assert got == want, f"draw {step}: device {got}, host {want}"
        ctx.append(int(got))
    assert s_dev.value == s_host.value
    assert len(set(ctx[32:])) > 16


def test_engine_sample_matches_host_logits(cuda_dev, qwen_weights):
    """sb_engine_sample (device candidates from the engine's own logits and
    token ids) draws what sb_sample_token draws on the same logits copied to
    the host, over 24 sampled steps."""
    L = sb200.lib()
    e = sb200.Engine(sb200.MODEL_QWEN, qwen_weights, 128)
    try:
        ids = [int(t) for t in sb200.synth_ids(8, V, 4242)]
        logits = np.zeros(V, dtype=np.float32)
        scratch = np.zeros(V, dtype=np.float32)
        s_eng, s_host = ctypes.c_uint32(1234), ctypes.c_uint32(1234)
        for p, t in enumerate(ids):
            e.forward(t, p, want_logits=(p == len(ids) - 1), logits_out=logits if p == len(ids) - 1 else None)
        for step in range(24):
            c = np.asarray(ids, dtype=np.int32)
            want = L.sb_sample_token(logits.ctypes.data, V, c.ctypes.data, len(ids), 0.7, 20, 0.8, 1.1,
                                     ctypes.byref(s_host), scratch.ctypes.data)
            got = e.sample(len(ids), s_eng)
            assert got == want, f"step {step}: engine {got}, host {want}"
            ids.append(got)
            e.forward(got, len(ids) - 1, True, logits)
    finally:
        e.close()
