"""CPU-side checks of the drop-in boundary: the C-ABI library loads, exports
every function include/switch_b200.h declares, embeds the five module images
(identical to the cubin files the reference hosts would load), and the
synthetic inputs are deterministic and in the reference layouts."""
import ctypes
import hashlib
import os
import re

import numpy as np
import pytest

import sb200

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "switch_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = sb200.lib()
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_module_images_embedded_and_on_disk():
    for name, path in sb200.CUBINS.items():
        img = sb200.module_image(name)
        assert len(img) > 1000
        with open(path, "rb") as f:
            disk = f.read()
        # the embedded image carries one trailing NUL (cuModuleLoadData of text images)
        assert img[: len(disk)] == disk


def test_cuda_calls_fail_loudly_without_a_driver():
    """With no GPU the product path raises; there is no CPU fallback."""
    if not sb200.driver_is_stub():
        pytest.skip("a real driver is present")
    with pytest.raises(sb200.SbError):
        sb200.init(0)


def test_synth_ids_deterministic():
    a = sb200.synth_ids(64, 151936, 5)
    assert a == sb200.synth_ids(64, 151936, 5)
    assert a != sb200.synth_ids(64, 151936, 6)
    assert all(0 <= t < 151936 for t in a)


def test_synth_uniform_and_normal():
    u = sb200.synth_uniform(1 << 16, -1.0, 1.0, 0)
    assert u.min() >= -1.0 and u.max() < 1.0 and abs(u.mean()) < 0.02
    h = sb200.synth_normal_h(1 << 16, 0.02, 0)
    f = h.view(np.float16).astype(np.float32)
    assert abs(f.std() - 0.02) < 0.001


def test_qwen_weight_layout(qwen_weights):
    """File size and fixed-offset fields match qwen_engine.c:60-75."""
    Q = sb200.QWEN
    assert os.path.getsize(qwen_weights) == Q["FILE_BYTES"]
    V, C, FC, CTX = Q["V"], Q["C"], Q["FC"], Q["CTX_FILE"]
    QKV = C + 2 * 128
    off_cos = V * C * 2
    lbase = off_cos + 2 * CTX * 32 * 4
    lstride = (C + QKV * C + QKV + C * C + C + 2 * FC * C + C * FC) * 2
    m = np.memmap(qwen_weights, dtype=np.uint8, mode="r")
    cos = np.frombuffer(m[off_cos: off_cos + CTX * 32 * 4], dtype=np.float32).reshape(CTX, 32)
    ang = np.outer(np.arange(CTX, dtype=np.float64), 1e6 ** (-2.0 * np.arange(32) / 64))
    np.testing.assert_allclose(cos, np.cos(ang).astype(np.float32), atol=1e-6)
    for l in (0, 23):
        b = lbase + l * lstride
        in_ln = np.frombuffer(m[b: b + C * 2], dtype=np.uint16)
        assert (in_ln == 0x3C00).all()  # RMSNorm weight 1.0
        post = b + (C + QKV * C + QKV + C * C) * 2
        assert (np.frombuffer(m[post: post + C * 2], dtype=np.uint16) == 0x3C00).all()
    lnf = lbase + 24 * lstride
    assert (np.frombuffer(m[lnf: lnf + C * 2], dtype=np.uint16) == 0x3C00).all()


def test_gpt2_weight_layout(gpt2_weights):
    G = sb200.GPT2
    assert os.path.getsize(gpt2_weights) == G["TOTAL_FLOATS"] * 4
    w = np.memmap(gpt2_weights, dtype=np.float32, mode="r")
    C = G["C"]
    lbase = G["V"] * C + G["CTX"] * C
    assert (w[lbase: lbase + C] == 1.0).all() and (w[lbase + C: lbase + 2 * C] == 0.0).all()
    assert (w[-2 * C: -C] == 1.0).all() and (w[-C:] == 0.0).all()
    assert abs(float(w[: 1 << 20].std()) - 0.02) < 0.001


def test_synth_weights_deterministic(tmp_path):
    a = tmp_path / "a.bin"
    sb200.synth_weights(sb200.MODEL_GPT2, a, 99)
    h1 = hashlib.sha256(open(a, "rb").read(1 << 24)).hexdigest()
    sb200.synth_weights(sb200.MODEL_GPT2, a, 99)
    assert hashlib.sha256(open(a, "rb").read(1 << 24)).hexdigest() == h1
