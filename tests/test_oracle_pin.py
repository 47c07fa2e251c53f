"""Pins the CPU oracle to the reference: bit-for-bit against the reference's
own C (oracle/_ref, built from the reference sources) where it is present,
against the committed golden fixtures (tests/golden/, generated from the
same reference C by tests/golden/make_golden.py) everywhere, and through the
reference's own harnesses (gpu_workload.c, gemv_test.c) run with the oracle
playing the device."""
import ctypes
import hashlib
import json
import os
import subprocess

import numpy as np
import pytest

import conftest
import orc
import sb200

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
need_ref = pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built (no reference sources)")
P = ctypes.c_void_p


def _load(fn):
    with open(os.path.join(GOLDEN, fn)) as f:
        return json.load(f)


def _hex(a):
    return [float(v).hex() for v in np.asarray(a, dtype=np.float32).ravel()]


# ------------------------------------------------------------------ fixtures (always)
def test_golden_gemv_h():
    g = _load("gemv_h.json")
    rng = np.random.default_rng(1)
    N, K = 64, 896
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16).view(np.uint16)
    W.ravel()[::53] = 0x0201
    x = rng.uniform(-1, 1, K).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float16).view(np.uint16)
    y = orc.gemv_h(W, x, orc.h2f(b))
    assert _hex(y) == g["y"]


@pytest.mark.parametrize("name", ["qwen", "gpt2"])
def test_golden_decode(name, qwen_weights, gpt2_weights):
    g = _load(f"{name}_decode.json")
    path = qwen_weights if name == "qwen" else gpt2_weights
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read(64 << 20)).hexdigest() == g["weights_sha256_first64MiB"], \
            "synthetic weight generator changed: regenerate the fixtures"
    vocab = sb200.QWEN["V"] if name == "qwen" else sb200.GPT2["V"]
    m = orc.Model(name, path, 16, vocab)
    try:
        for p, (t, st) in enumerate(zip(g["ids"], g["steps"])):
            lg = m.forward(t, p, True)
            assert int(np.argmax(lg)) == st["argmax"]
            assert _hex(lg[:16]) == st["first16"]
            assert hashlib.sha256(lg.tobytes()).hexdigest() == st["sha256"]
    finally:
        m.close()


# ------------------------------------------------------------------ reference C (when built)
@need_ref
def test_h2f_all_bit_patterns():
    L = orc.ref_lib("qwen")
    bits = np.arange(65536, dtype=np.uint16)
    ref = np.array([L.ref_h2f(int(b)) for b in bits], dtype=np.float32)
    ours = np.array([orc.oracle().orc_h2f(int(b)) for b in bits], dtype=np.float32)
    assert np.array_equal(ref.view(np.uint32), ours.view(np.uint32))
    fin = np.isfinite(ref)
    assert np.array_equal(orc.h2f(bits)[fin], ref[fin])


@need_ref
@pytest.mark.parametrize("N,K", [(37, 896), (5, 4864), (64, 8)])
def test_gemv_h_bitwise(N, K):
    L = orc.ref_lib("qwen")
    W = sb200.synth_normal_h(N * K, 0.02, N).reshape(N, K)
    W.ravel()[::31] = 0x0101
    x = sb200.synth_uniform(K, -1, 1, K)
    b = sb200.synth_normal_h(N, 0.02, 1)
    ref = np.zeros(N, dtype=np.float32)
    L.ref_gemv_h(W.ctypes.data_as(P), x.ctypes.data_as(P), b.ctypes.data_as(P), ref.ctypes.data_as(P), K, N)
    assert np.array_equal(orc.gemv_h(W, x, orc.h2f(b)), ref)


@need_ref
def test_rms_and_gemv_f32_and_ln_bitwise():
    Lq, Lg = orc.ref_lib("qwen"), orc.ref_lib("gpt2")
    x = sb200.synth_uniform(896, -3, 3, 1)
    w = sb200.synth_normal_h(896, 1.0, 2)
    ref = np.zeros(896, dtype=np.float32)
    Lq.ref_rms(x.ctypes.data_as(P), w.ctypes.data_as(P), ref.ctypes.data_as(P), 896)
    assert np.array_equal(orc.rmsnorm(x, w, 1e-6), ref)
    N, K = 50, 768
    W = sb200.synth_uniform(N * K, -0.1, 0.1, 3).reshape(N, K)
    v = sb200.synth_uniform(K, -1, 1, 4)
    bb = sb200.synth_uniform(N, -0.1, 0.1, 5)
    ref = np.zeros(N, dtype=np.float32)
    Lg.ref_gemv(W.ctypes.data_as(P), v.ctypes.data_as(P), bb.ctypes.data_as(P), ref.ctypes.data_as(P), K, N)
    assert np.array_equal(orc.gemv_f32(W, v, bb), ref)
    lw = sb200.synth_uniform(768, 0.5, 1.5, 6)
    lb = sb200.synth_uniform(768, -0.2, 0.2, 7)
    ref = np.zeros(768, dtype=np.float32)
    Lg.ref_ln(v.ctypes.data_as(P), lw.ctypes.data_as(P), lb.ctypes.data_as(P), ref.ctypes.data_as(P))
    assert np.array_equal(orc.layernorm(v, lw, lb, 1e-5), ref)


@need_ref
@pytest.mark.parametrize("name", ["qwen", "gpt2"])
def test_decode_forward_bitwise(name, qwen_weights, gpt2_weights):
    """The oracle's restated cpu_forward equals the reference's bit for bit
    (logits and residual) over several positions, including a prompt step
    without logits."""
    path = qwen_weights if name == "qwen" else gpt2_weights
    vocab = sb200.QWEN["V"] if name == "qwen" else sb200.GPT2["V"]
    C = sb200.QWEN["C"] if name == "qwen" else sb200.GPT2["C"]
    L = orc.ref_lib(name)
    getattr(L, f"ref_{name}_load")(path.encode())
    m = orc.Model(name, path, 16, vocab)
    ids = sb200.synth_ids(5, vocab, 77)
    try:
        for p, t in enumerate(ids):
            want_logits = p != 1
            ref = np.zeros(vocab, dtype=np.float32)
            getattr(L, f"ref_{name}_forward")(t, p, 1 if want_logits else 0, ref.ctypes.data_as(P))
            got = m.forward(t, p, want_logits)
            rres = np.zeros(C, dtype=np.float32)
            getattr(L, f"ref_{name}_residual")(rres.ctypes.data_as(P))
            ores = np.ctypeslib.as_array(ctypes.cast(getattr(orc.oracle(), f"orc_{name}_residual")(m.h),
                                                     ctypes.POINTER(ctypes.c_float)), shape=(C,))
            assert np.array_equal(ores, rres), f"residual differs at pos {p}"
            if want_logits:
                assert np.array_equal(got, ref), f"logits differ at pos {p}"
    finally:
        m.close()


@need_ref
def test_reference_sgemm_harness_accepts_oracle(tmp_path):
    """gpu_workload.c itself (its CPU triple loop and tolerance, sizes
    256/512/1024) accepts the oracle's SGEMM as the device result, and flags a
    planted 10% error in one cell."""
    mod = tmp_path / "m.ptx"
    mod.write_text("")
    exe = os.path.join(orc.REF_DIR, "gpu_workload_emu")
    out = subprocess.run([exe, "--json", str(mod)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0
    j = json.loads(out.stdout)
    assert j["done"] is True and set(j["kernels"].values()) == {"CORRECT"} and len(j["kernels"]) == 4
    env = dict(os.environ, ORC_EMU_PLANT="1")
    out = subprocess.run([exe, "--json", str(mod)], capture_output=True, text=True, timeout=300, env=env)
    assert set(json.loads(out.stdout)["kernels"].values()) == {"WRONG"}


@need_ref
def test_reference_gemv_harness_accepts_oracle(tmp_path):
    """gemv_test.c (its serial golden loop, LCG seed 42, 1e-4 rel+abs
    tolerance) accepts the oracle's FP32 GEMV; exit status 1 on a planted error."""
    mod = tmp_path / "m.ptx"
    mod.write_text("")
    exe = os.path.join(orc.REF_DIR, "gemv_test_emu")
    out = subprocess.run([exe, str(mod), "2048", "1024"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and "GEMV_TEST_DONE" in out.stdout
    assert out.stdout.count("CORRECT") == 3
    env = dict(os.environ, ORC_EMU_PLANT="1")
    out = subprocess.run([exe, str(mod), "2048", "1024"], capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 1 and "GEMV_TEST_FAILED" in out.stdout


def test_oracle_greedy_loop_shape(gpt2_weights):
    """orc.greedy follows the reference's prime-then-generate loop: n_prompt
    forwards (logits only on the last), then n_gen forwards, n_gen+1 new ids."""
    m = orc.Model("gpt2", gpt2_weights, 16, sb200.GPT2["V"])
    try:
        ids, steps = orc.greedy(m, [1, 2, 3], 4)
        assert len(ids) == 3 + 4 + 1 and len(steps) == 5
        assert ids[3] == int(np.argmax(steps[0]))
    finally:
        m.close()
