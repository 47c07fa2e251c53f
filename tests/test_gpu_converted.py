"""A converted checkpoint runs: sb_convert turns a seeded synthetic Hugging
Face checkpoint (every tensor of the model; Qwen BF16, GPT-2 F32) into the
engine's weight file, and the engine's teacher-forced logits on that file
match the oracle's restatement of the reference cpu_forward on the same
file (relative Frobenius <= 2e-3 per step, same argmax)."""
import os
import sys

import numpy as np
import pytest

import orc
import sb200
import sb_convert

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import conv_synth  # noqa: E402

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3


def _rel(a, b):
    return float(np.linalg.norm((a - b).astype(np.float64)) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


@pytest.mark.parametrize("model", ["qwen", "gpt2"])
def test_converted_checkpoint_decodes(cuda_dev, tmp_path, model):
    src, dst = str(tmp_path / "model.safetensors"), str(tmp_path / "model.bin")
    (conv_synth.write_qwen if model == "qwen" else conv_synth.write_gpt2)(src, 20261221)
    sb_convert.convert(model, src, dst)
    os.unlink(src)
    mid, vocab = ((sb200.MODEL_QWEN, sb200.QWEN["V"]) if model == "qwen" else (sb200.MODEL_GPT2, sb200.GPT2["V"]))
    ids = sb200.synth_ids(6, vocab, 3)
    eng = sb200.Engine(mid, dst, 32)
    ref = orc.Model(model, dst, 32, vocab)
    try:
        for p, t in enumerate(ids):
            got = np.zeros(vocab, dtype=np.float32)
            eng.forward(t, p, True, got)
            want = ref.forward(t, p, True)
            assert np.isfinite(got).all()
            assert _rel(got, want) <= LOGIT_TOL, f"pos {p}: rel err {_rel(got, want):.2e}"
            assert int(np.argmax(got)) == int(np.argmax(want))
    finally:
        eng.close()
        ref.close()
