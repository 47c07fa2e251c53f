"""Converters (sb_convert): byte-identical engine files versus the reference's
gpu-llm/tools/conv_qwen.py and conv_gpt2.py, pinned by tests/golden/convert.json
(made by tests/golden/make_conv_golden.py from the reference scripts), plus
the error cases the reference scripts reject (missing tensor, wrong shape,
non-F32 GPT-2 source) and an exact check of the FP16 rounding itself."""
import json
import os
import struct
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import conv_synth  # noqa: E402
import make_conv_golden  # noqa: E402
import sb_convert  # noqa: E402

GOLD = json.load(open(os.path.join(HERE, "golden", "convert.json")))


@pytest.mark.parametrize("model", ["qwen", "gpt2"])
def test_matches_reference_converter(model, tmp_path):
    g = GOLD[model]
    src, dst = str(tmp_path / "m.safetensors"), str(tmp_path / "m.bin")
    (conv_synth.write_qwen if model == "qwen" else conv_synth.write_gpt2)(src, g["seed"])
    assert make_conv_golden.file_digest(src)[1] == g["checkpoint_sha256"], "synthetic checkpoint generator drifted"
    n = sb_convert.convert(model, src, dst)
    size, sha, blocks = make_conv_golden.file_digest(dst)
    assert n == size == g["bytes"]
    if sha != g["sha256"]:
        bad = [i for i, (a, b) in enumerate(zip(blocks, g["block_sha256"])) if a != b]
        pytest.fail(f"{model}: output differs from the reference converter's in 64 MiB blocks {bad}")


def test_gpt2_prefixed_names(tmp_path):
    """Checkpoints saved from GPT2LMHeadModel name the tensors
    'transformer.h.0...': same values, so the same output bytes."""
    g = GOLD["gpt2"]
    src, dst = str(tmp_path / "p.safetensors"), str(tmp_path / "p.bin")
    conv_synth.write(src, [("transformer." + n, shp) for n, shp in conv_synth.gpt2_tensors()], "F32", g["seed"])
    sb_convert.convert("gpt2", src, dst)
    assert make_conv_golden.file_digest(dst)[1] == g["sha256"]


def test_qwen_f16_source_is_copied_exactly(tmp_path):
    """An F16 checkpoint (conv_qwen.py:38-39 widens it to FP32 and rounds
    back): every weight lands in the file bit for bit, at the engine's
    offsets (embedding, fused q|k|v rows and biases, gate|up rows, down
    rows, final norm)."""
    V, C, NL, QKV, FC, CTX, HD = 151936, 896, 24, 1152, 4864, 8192, 64
    src, dst = str(tmp_path / "q16.safetensors"), str(tmp_path / "q16.bin")
    conv_synth.write(src, conv_synth.qwen_tensors(), "F16", 20261231)
    sb_convert.convert("qwen", src, dst)
    st = sb_convert.SafeTensors(src)
    out = np.memmap(dst, dtype=np.uint8, mode="r")

    def raw(*names):
        return np.concatenate([np.ascontiguousarray(st.raw(n)).view(np.uint8).ravel() for n in names])

    lbase = V * C * 2 + 2 * CTX * (HD // 2) * 4
    lstride = (C + QKV * C + QKV + C * C + C + 2 * FC * C + C * FC) * 2
    assert np.array_equal(out[:V * C * 2], raw("model.embed_tokens.weight"))
    for layer in (0, 13, NL - 1):
        p, base = f"model.layers.{layer}.", lbase + layer * lstride
        qkvw = base + C * 2
        qkvb = qkvw + QKV * C * 2
        post = qkvb + QKV * 2 + C * C * 2
        gateup = post + C * 2
        down = gateup + 2 * FC * C * 2
        assert np.array_equal(out[base:qkvw], raw(p + "input_layernorm.weight"))
        assert np.array_equal(out[qkvw:qkvb], raw(p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                                                  p + "self_attn.v_proj.weight"))
        assert np.array_equal(out[qkvb:qkvb + QKV * 2], raw(p + "self_attn.q_proj.bias", p + "self_attn.k_proj.bias",
                                                            p + "self_attn.v_proj.bias"))
        assert np.array_equal(out[gateup:down], raw(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"))
        assert np.array_equal(out[down:down + C * FC * 2], raw(p + "mlp.down_proj.weight"))
    lnf = lbase + NL * lstride
    assert np.array_equal(out[lnf:], raw("model.norm.weight"))


def _tiny_safetensors(path, tensors):
    """tensors: {name: (dtype string, ndarray of the stored type)}"""
    header, off, blobs = {}, 0, []
    for name, (dt, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def test_widen_and_round_fp16_exact():
    # BF16 -> FP32 is a 16-bit shift; FP32 -> FP16 rounds to nearest even and keeps subnormals
    bits = np.array([0x3F80, 0xBF80, 0x3800, 0x3380, 0x0000, 0x8000, 0x477F], dtype=np.uint16)
    f = sb_convert.widen(bits)
    assert f.tolist() == [1.0, -1.0, 2.0 ** -15, 2.0 ** -24, 0.0, -0.0, 65280.0]
    h = f.astype(np.float16)
    assert h.view(np.uint16).tolist() == [0x3C00, 0xBC00, 0x0200, 0x0001, 0x0000, 0x8000, 0x7BF8]
    # ties to even at the FP16 grid: 1 + 2^-11 -> 1.0, 1 + 3*2^-11 -> 1 + 2^-9
    t = np.array([1 + 2.0 ** -11, 1 + 3 * 2.0 ** -11], dtype=np.float32).astype(np.float16)
    assert t.view(np.uint16).tolist() == [0x3C00, 0x3C02]


def test_missing_tensor_rejected_before_writing(tmp_path):
    src, dst = str(tmp_path / "x.safetensors"), str(tmp_path / "x.bin")
    _tiny_safetensors(src, {"model.norm.weight": ("F32", np.ones(896, np.float32))})
    with pytest.raises(sb_convert.ConvertError, match="embed_tokens"):
        sb_convert.convert("qwen", src, dst)
    assert not os.path.exists(dst) and not os.path.exists(dst + ".partial")


def test_wrong_shape_rejected(tmp_path):
    src, dst = str(tmp_path / "x.safetensors"), str(tmp_path / "x.bin")
    _tiny_safetensors(src, {"wte.weight": ("F32", np.zeros((10, 768), np.float32))})
    with pytest.raises(sb_convert.ConvertError, match="shape"):
        sb_convert.convert("gpt2", src, dst)


def test_gpt2_needs_f32(tmp_path):
    src, dst = str(tmp_path / "x.safetensors"), str(tmp_path / "x.bin")
    _tiny_safetensors(src, {"wte.weight": ("F16", np.zeros((50257, 768), np.float16))})
    with pytest.raises(sb_convert.ConvertError, match="F32"):
        sb_convert.convert("gpt2", src, dst)


def test_cli_usage_and_failure(tmp_path, capsys):
    assert sb_convert.main(["sb_convert.py"]) == 2
    assert sb_convert.main(["sb_convert.py", "qwen", str(tmp_path / "absent.safetensors"),
                            str(tmp_path / "o.bin")]) == 1
    assert "conversion failed" in capsys.readouterr().err
