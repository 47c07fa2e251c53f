"""The reference-compatible command-line hosts on the GPU: the Qwen engine's
`--serve` wire protocol (gpu-llm/engine/qwen_engine.c:406-444, read by
gpu-llm/server/qwen_serve.py), `--ids`/`--gen` greedy generation into
out.ids for both engines (qwen_engine.c:523-556, gpt2_engine.c:540-573),
and gemv_test's verdict lines (gpu-llm/harness/gemv_test.c).  Each output
is checked against the oracle's restatement of the reference's greedy loop
on the same weight file."""
import os
import struct
import subprocess

import numpy as np
import pytest

import orc
import sb200

pytestmark = pytest.mark.gpu
BIN = os.path.join(os.path.dirname(sb200.__file__), "bin")
QW_EOS = (151643, 151645)
G2_EOS = (50256,)


def _write_ids(path, ids):
    with open(path, "wb") as f:
        f.write(struct.pack("<I", len(ids)))
        f.write(struct.pack(f"<{len(ids)}I", *ids))


def _read_ids(path):
    with open(path, "rb") as f:
        n = struct.unpack("<I", f.read(4))[0]
        return list(struct.unpack(f"<{n}I", f.read(4 * n)))


def _oracle_greedy(name, weights, vocab, prompt, n_gen, eos):
    ref = orc.Model(name, weights, len(prompt) + n_gen + 8, vocab)
    try:
        ids, _ = orc.greedy(ref, prompt, n_gen, eos)
    finally:
        ref.close()
    return ids


def test_qwen_serve_two_requests(cuda_dev, qwen_weights):
    """Two framed requests on one process (u32 T, T x u32 ids, u32 max_gen ->
    u32 M, M x u32 ids: prompt echo + generation), greedy; each reply equals
    the oracle's greedy loop, and the second request is not disturbed by the
    first one's cache."""
    V = sb200.QWEN["V"]
    reqs = [(sb200.synth_ids(11, V, 501), 7), (sb200.synth_ids(5, V, 502), 12)]
    stdin = b"".join(struct.pack("<I", len(p)) + struct.pack(f"<{len(p)}I", *p) + struct.pack("<I", g)
                     for p, g in reqs)
    out = subprocess.run([os.path.join(BIN, "qwen_engine"), "--weights", str(qwen_weights), "--serve", "--greedy",
                          "--ctx", "256"], input=stdin, capture_output=True, timeout=300)
    assert out.returncode == 0, out.stderr.decode()[-800:]
    buf = out.stdout
    for prompt, maxg in reqs:
        m = struct.unpack("<I", buf[:4])[0]
        got = list(struct.unpack(f"<{m}I", buf[4:4 + 4 * m]))
        buf = buf[4 + 4 * m:]
        want = _oracle_greedy("qwen", qwen_weights, V, prompt, maxg, QW_EOS)
        assert got == want
    assert buf == b""  # nothing else on stdout: banners go to stderr
    assert out.stderr.decode().count("serve: T=") == 2


@pytest.mark.parametrize("model", ["qwen", "gpt2"])
def test_engine_cli_greedy_out_ids(cuda_dev, qwen_weights, gpt2_weights, tmp_path, model):
    """`--ids F --gen N` writes prompt + generated ids to out.ids in the
    working directory, prints the reference's summary lines and ENGINE_DONE."""
    if model == "qwen":
        exe, w, V, eos, extra = "qwen_engine", qwen_weights, sb200.QWEN["V"], QW_EOS, ["--greedy", "--ctx", "128"]
    else:
        exe, w, V, eos, extra = "gpt2_engine", gpt2_weights, sb200.GPT2["V"], G2_EOS, ["--ctx", "128"]
    prompt = sb200.synth_ids(9, V, 777)
    _write_ids(tmp_path / "p.ids", prompt)
    out = subprocess.run([os.path.join(BIN, exe), "--weights", str(w), "--ids", "p.ids", "--gen", "10"] + extra,
                         capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert out.returncode == 0, out.stderr[-800:]
    assert "prompt: 9 token(s)" in out.stdout and out.stdout.rstrip().endswith("ENGINE_DONE")
    assert _read_ids(tmp_path / "out.ids") == _oracle_greedy(model, w, V, prompt, 10, eos)


def test_qwen_cli_sampled_out_ids(cuda_dev, qwen_weights, tmp_path):
    """Without --greedy the engine samples with the reference's settings
    (qwen_engine.c:375-399: penalty 1.1, temperature 0.7, top-k 20, top-p
    0.8, xorshift seeded 1234), its top-20 picked on the device.  out.ids
    equals the reference's prime-then-sample loop run on the same engine's
    logits (copied to the host each step) and drawn by the reference's own
    sample_token where oracle/_ref is built (else by sb_sample_token, which
    tests/test_cpu_sampler.py pins to it).  The logits themselves are
    checked against the oracle in tests/test_gpu_engine.py; sampling from
    CPU-oracle logits instead would make the comparison depend on near-ties
    among the top candidates."""
    import ctypes

    V = sb200.QWEN["V"]
    prompt = sb200.synth_ids(9, V, 778)
    _write_ids(tmp_path / "p.ids", prompt)
    out = subprocess.run([os.path.join(BIN, "qwen_engine"), "--weights", str(qwen_weights), "--ids", "p.ids", "--gen",
                          "12", "--ctx", "128"], capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert out.returncode == 0, out.stderr[-800:]
    got = _read_ids(tmp_path / "out.ids")
    if orc.ref_available():
        refl = orc.ref_lib("qwen")
        refl.ref_sampler_seed(1234)

        def draw(logits, ids):
            c = np.asarray(ids, dtype=np.int32)
            return refl.ref_sample_token(logits.ctypes.data_as(ctypes.c_void_p), c.ctypes.data_as(ctypes.c_void_p),
                                         len(ids))
    else:
        state, scratch = ctypes.c_uint32(1234), np.zeros(V, dtype=np.float32)

        def draw(logits, ids):
            c = np.asarray(ids, dtype=np.int32)
            return sb200.lib().sb_sample_token(logits.ctypes.data, V, c.ctypes.data, len(ids), 0.7, 20, 0.8, 1.1,
                                               ctypes.byref(state), scratch.ctypes.data)
    e = sb200.Engine(sb200.MODEL_QWEN, qwen_weights, 128)
    try:
        ids, logits = list(prompt), np.zeros(V, dtype=np.float32)
        for p, t in enumerate(prompt):
            e.forward(t, p, p == len(prompt) - 1, logits if p == len(prompt) - 1 else None)
        nxt = draw(logits, ids)
        ids.append(nxt)
        for _ in range(12):
            if nxt in QW_EOS:
                break
            e.forward(nxt, len(ids) - 1, True, logits)
            nxt = draw(logits, ids)
            ids.append(nxt)
    finally:
        e.close()
    assert got == ids
    assert len(set(got[9:])) > 3  # sampled, not a repeated argmax


def test_gemv_test_cli(cuda_dev):
    """gemv_test <module> N K: every kernel of the M0 module CORRECT against
    the harness's CPU loop, then GEMV_TEST_DONE."""
    out = subprocess.run([os.path.join(BIN, "gemv_test"), sb200.CUBINS["gemv"], "1000", "772"], capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-800:]
    for name in ("gemv", "gemv4", "gemv_warp"):
        assert f"{name}: CORRECT" in out.stdout
    assert out.stdout.rstrip().endswith("GEMV_TEST_DONE")


def test_qwen_selftest_and_debug(cuda_dev, qwen_weights, tmp_path):
    """--selftest N compares the engine's logits at position N-1 with the
    serial CPU forward written in the host (not the test oracle), as the
    reference's selftest does; --debug adds the layer-0 stage dumps of
    position 0 from a per-stage GPU pass (g.*) and from the CPU forward (c.*)."""
    V = sb200.QWEN["V"]
    _write_ids(tmp_path / "p.ids", sb200.synth_ids(4, V, 31))
    out = subprocess.run([os.path.join(BIN, "qwen_engine"), "--weights", str(qwen_weights), "--ids", "p.ids",
                          "--selftest", "4", "--debug", "--greedy", "--gen", "2", "--ctx", "64"],
                         capture_output=True, text=True, timeout=600, cwd=tmp_path)
    assert out.returncode == 0, out.stderr[-800:]
    o = out.stdout
    assert "selftest: comparing GPU vs serial-CPU logits at position 3" in o
    assert "SELFTEST: PASS" in o and "MATCH" in o
    err = float(o.split("max |gpu-cpu| logit err:")[1].split()[0])
    assert err < 0.05, o
    for tag in ("g.ln1", "g.qkv", "g.scores", "g.probs", "g.attnout", "g.res1", "g.gate", "g.swiglu", "g.res2",
                "c.embed", "c.ln1", "c.qkv", "c.ao", "c.res1"):
        assert tag in o, tag
    assert o.rstrip().endswith("ENGINE_DONE")


@pytest.mark.parametrize("model", ["qwen", "gpt2"])
def test_ptx_module_path(cuda_dev, qwen_weights, gpt2_weights, tmp_path, model):
    """--ptx M decodes through module M's drop-in kernels with the
    reference's per-stage launches (this package's cubin is passed, as an
    operator would pass theirs); out.ids equals the oracle's greedy loop."""
    if model == "qwen":
        exe, w, V, eos, extra = "qwen_engine", qwen_weights, sb200.QWEN["V"], QW_EOS, ["--greedy", "--ctx", "64"]
    else:
        exe, w, V, eos, extra = "gpt2_engine", gpt2_weights, sb200.GPT2["V"], G2_EOS, ["--ctx", "64"]
    prompt = sb200.synth_ids(6, V, 4242)
    _write_ids(tmp_path / "p.ids", prompt)
    mod = sb200.CUBINS[model]
    out = subprocess.run([os.path.join(BIN, exe), "--weights", str(w), "--ptx", mod, "--ids", "p.ids", "--gen", "6"]
                         + extra, capture_output=True, text=True, timeout=600, cwd=tmp_path)
    assert out.returncode == 0, out.stderr[-800:]
    assert f"module {mod}" in out.stdout and "per-stage module kernels" in out.stdout
    assert _read_ids(tmp_path / "out.ids") == _oracle_greedy(model, w, V, prompt, 6, eos)


@pytest.mark.parametrize("fused", [False, True])
def test_gpt2_selftest_trace_ptx(cuda_dev, gpt2_weights, tmp_path, fused):
    """GPT-2's selftest with the reference's per-layer residual trace of
    position 0, through --ptx (and --fused: gemv_warp_b launches)."""
    _write_ids(tmp_path / "p.ids", sb200.synth_ids(5, sb200.GPT2["V"], 55))
    cmd = [os.path.join(BIN, "gpt2_engine"), "--weights", str(gpt2_weights), "--ptx", sb200.CUBINS["gpt2"], "--ids",
           "p.ids", "--selftest", "5", "--debug", "--gen", "2", "--ctx", "64"] + (["--fused"] if fused else [])
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=tmp_path)
    assert out.returncode == 0, out.stderr[-800:]
    o = out.stdout
    traces = [ln for ln in o.splitlines() if ln.strip().startswith("trace p0 L")]
    assert len(traces) == 12
    assert max(float(ln.split("max|d|=")[1].split()[0]) for ln in traces) < 1e-2
    assert "SELFTEST: PASS" in o and "g.gelu" in o and "c.gelu" in o
