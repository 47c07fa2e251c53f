"""The host sampler sb_sample_token against the reference's own sample_token
(gpu-llm/engine/qwen_engine.c:369-399, compiled unmodified into
oracle/_ref/libref_qwen.so): repetition penalty 1.1 over the context,
temperature 0.7, top-k 20 by repeated first-index argmax, clamped-exp
softmax, top-p 0.8, and a draw from the engine's xorshift state seeded 1234.
Given the same logits, context and state, both must draw the same token --
checked over 256 consecutive draws whose context grows with the drawn ids,
so repeated ids are penalised repeatedly, as in the reference's loop."""
import ctypes
import os

import numpy as np
import pytest

import orc
import sb200

V = 151936


def _logits(rng, ctx):
    """Realistic-looking logits: a N(0, 1.5) floor, a few strong candidates
    (so top-p keeps several), some of them ids already in the context (so
    the penalty changes the ranking), and exact ties among the leaders (so
    the first-index rule decides)."""
    w = rng.normal(0.0, 1.5, V).astype(np.float32)
    lead = rng.integers(0, V, 12)
    w[lead] = rng.uniform(6.0, 9.0, 12).astype(np.float32)
    if ctx:
        rep = rng.choice(ctx, size=min(4, len(ctx)), replace=False)
        w[rep] = rng.uniform(6.0, 9.5, len(rep)).astype(np.float32)
        w[rep[0]] = -w[rep[0]]  # a negative, penalised by multiplication
    w[lead[1]] = w[lead[0]]
    return w


@pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
def test_sampler_matches_reference_256_draws():
    ref = orc.ref_lib("qwen")
    ref.ref_sampler_seed(1234)
    state = ctypes.c_uint32(1234)
    scratch = np.zeros(V, dtype=np.float32)
    rng = np.random.default_rng(99)
    ctx = [int(t) for t in sb200.synth_ids(32, V, 1000)]
    L = sb200.lib()
    for step in range(256):
        w = _logits(rng, ctx)
        c = np.asarray(ctx, dtype=np.int32)
        want = ref.ref_sample_token(w.ctypes.data_as(ctypes.c_void_p), c.ctypes.data_as(ctypes.c_void_p), len(ctx))
        got = L.sb_sample_token(w.ctypes.data_as(ctypes.c_void_p), V, c.ctypes.data_as(ctypes.c_void_p), len(ctx),
                                ctypes.c_float(0.7), 20, ctypes.c_float(0.8), ctypes.c_float(1.1),
                                ctypes.byref(state), scratch.ctypes.data_as(ctypes.c_void_p))
        assert got == want, f"draw {step}: sb_sample_token {got}, reference {want}"
        ctx.append(int(got))
    # the draws were not all the top candidate: the distribution was sampled
    assert len(set(ctx[32:])) > 16


@pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
def test_topk_restatement_and_host_draw_match_reference():
    """The float32 restatement of steps 1-3 that the GPU sampler test uses
    as its oracle, followed by sb_sample_topk (steps 4-6), draws what the
    reference's sample_token draws: 64 consecutive draws."""
    from test_gpu_sampler import _host_topk, _logits
    ref = orc.ref_lib("qwen")
    ref.ref_sampler_seed(1234)
    state = ctypes.c_uint32(1234)
    rng = np.random.default_rng(5)
    ctx = [int(t) for t in sb200.synth_ids(32, V, 1000)]
    for step in range(64):
        w = _logits(rng, ctx)
        c = np.asarray(ctx, dtype=np.int32)
        want = ref.ref_sample_token(w.ctypes.data_as(ctypes.c_void_p), c.ctypes.data_as(ctypes.c_void_p), len(ctx))
        idx, val = _host_topk(w, ctx, 20)
        got = sb200.sample_topk(idx, val, 0.8, state)
        assert got == want, f"draw {step}: {got} against the reference's {want}"
        ctx.append(int(got))

