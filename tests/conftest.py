"""Shared pytest setup: the `gpu` marker, import paths, and session-wide
synthetic weight files in the reference layouts."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "switch-l4t-gpu_b200")
for p in (PKG, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

QWEN_SEED = 20261201
GPT2_SEED = 20261202


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


# Parity margins: the engine tests record their worst per-step error next to
# the bar it must stay under; the session summary prints them, so a drift
# toward a bar is visible in a passing run.
MARGINS = {}


def record_margin(name, err, bar):
    prev = MARGINS.get(name)
    if prev is None or err > prev[0]:
        MARGINS[name] = (float(err), float(bar))


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not MARGINS:
        return
    terminalreporter.section("parity margins (worst error / bar)")
    for name in sorted(MARGINS):
        err, bar = MARGINS[name]
        terminalreporter.write_line(f"{name}: {err:.3e} / {bar:.0e}  ({100 * err / bar:.1f}% of the bar)")


def _weights_dir():
    d = os.environ.get("SB_WEIGHTS_DIR") or ("/dev/shm/sb200_weights" if os.path.isdir("/dev/shm") else "/tmp/sb200_weights")
    os.makedirs(d, exist_ok=True)
    return d


def _synth(model, name, seed, size):
    import sb200
    path = os.path.join(_weights_dir(), f"{name}_{seed}.bin")
    if not (os.path.exists(path) and os.path.getsize(path) == size):
        tmp = path + f".tmp{os.getpid()}"
        n = sb200.synth_weights(model, tmp, seed)
        assert n == size
        os.replace(tmp, path)
    return path


@pytest.fixture(scope="session")
def qwen_weights():
    import sb200
    return _synth(sb200.MODEL_QWEN, "qwen", QWEN_SEED, sb200.QWEN["FILE_BYTES"])


@pytest.fixture(scope="session")
def gpt2_weights():
    import sb200
    return _synth(sb200.MODEL_GPT2, "gpt2", GPT2_SEED, sb200.GPT2["TOTAL_FLOATS"] * 4)


@pytest.fixture(scope="session")
def cuda_dev():
    """torch on cuda:0 with the primary context current on this thread."""
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("GPU test without a CUDA device")
    torch.cuda.init()
    torch.zeros(1, device="cuda")
    import sb200
    sb200.init(0)
    return torch.device("cuda:0")
