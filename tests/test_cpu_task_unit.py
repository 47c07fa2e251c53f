"""Task-queue consumer (task_unit): the contract of the reference's
deploy/cluster/gpu_task_example.py, driven by fake harnesses that replay the
output formats of this package's gpu_workload (JSON and text), plus one GPU
test that runs the real harness."""
import json
import os
import stat
from pathlib import Path

import pytest

import task_unit

PKG = Path(task_unit.__file__).resolve().parent


def _json_out(**over):
    d = {"ptx": "/x/lib/switch_gpu.cubin",
         "kernels": {"sgemm": "CORRECT", "sgemm_naive": "CORRECT", "sgemm_tiled4": "CORRECT",
                     "sgemm_opt": "CORRECT", "sgemm_b200": "CORRECT"},
         "sgemm": [{"n": 256, "ms": 0.031, "gflops": 1076.8}, {"n": 512, "ms": 0.049, "gflops": 5478.2},
                   {"n": 1024, "ms": 0.105, "gflops": 20452.4}],
         "membw_gbps": 6917.2, "membw_bytes": 8589934592, "device": "NVIDIA B200", "sm_count": 148,
         "fp32_peak_gflops_at_max_clock": 74449.9, "done": True}
    d.update(over)
    return json.dumps(d)


TEXT_OUT = """sgemm 256: CORRECT
sgemm_naive 256: CORRECT (0 bad cells)
sgemm_tiled4 256: CORRECT
sgemm 256x256x256: 0.031 ms/iter, 1076.8 GFLOPS
sgemm_tiled4 256x256x256: 0.031 ms/iter, 1075.0 GFLOPS
sgemm 512x512x512: 0.049 ms/iter, 5478.2 GFLOPS
sgemm 1024x1024x1024: 0.105 ms/iter, 20452.4 GFLOPS
membw read (2048 MiB x4): 0.001 s, 6886.8 GB/s
WORKLOAD_DONE
"""


def _home(tmp_path, script, module="switch_gpu_native.ptx"):
    """A GPU home whose gpu_workload is the given shell script body."""
    home = tmp_path / "home"
    home.mkdir(parents=True)
    exe = home / "gpu_workload"
    exe.write_text("#!/bin/sh\n" + script)
    exe.chmod(exe.stat().st_mode | stat.S_IXUSR)
    (home / module).write_bytes(b"module image")
    return home


def _printer(text):
    return "cat <<'EOF'\n" + text + "\nEOF\n"


def test_json_unit(tmp_path):
    r = task_unit.run_unit(_home(tmp_path, _printer(_json_out())))
    assert r["correct"] is True and r["device"] == "NVIDIA B200"
    assert r["gflops"] == {"256": 1076.8, "512": 5478.2, "1024": 20452.4} and r["gbps"] == 6917.2
    assert "sgemm_b200" in r["kernels_verified"]
    task_unit.verify_unit(r)


def test_text_fallback_for_harness_without_json(tmp_path):
    # an old harness takes --json for the module path, fails, and prints no JSON
    script = 'if [ "$1" = "--json" ]; then echo "cannot read --json" >&2; exit 1; fi\n' + _printer(TEXT_OUT)
    r = task_unit.run_unit(_home(tmp_path, script, module="switch_gpu.cubin"))
    assert r["gflops"]["1024"] == 20452.4 and r["gbps"] == 6886.8
    assert r["kernels_verified"] == ["sgemm", "sgemm_naive", "sgemm_tiled4"]


@pytest.mark.parametrize("out, msg", [
    (_json_out(kernels={"sgemm": "CORRECT", "sgemm_opt": "WRONG"}), "golden-model"),
    (_json_out(done=False), "truncated"),
    (_json_out(kernels={"sgemm_opt": "CORRECT"}), "kernels.sgemm"),
    (_json_out(sgemm=[{"n": 256, "gflops": 1.0e3}]), "size"),
    (_json_out(membw_gbps=12000.0), "gbps"),
    (_json_out(sgemm=[{"n": 256, "gflops": 1e3}, {"n": 512, "gflops": 5e3}, {"n": 1024, "gflops": 90000.0}]),
     "gflops\\[1024\\]"),
    # above the harness's own clock-derived peak (x 1.02), though under the static bound
    (_json_out(fp32_peak_gflops_at_max_clock=15000.0), "gflops\\[1024\\]"),
    (_json_out()[:-20], "invalid --json"),
])
def test_json_rejections(tmp_path, out, msg):
    with pytest.raises(task_unit.UnitError, match=msg):
        task_unit.run_unit(_home(tmp_path, _printer(out)))


@pytest.mark.parametrize("out, msg", [
    (TEXT_OUT.replace("WORKLOAD_DONE", ""), "WORKLOAD_DONE"),
    (TEXT_OUT.replace("sgemm_tiled4 256: CORRECT", "sgemm_tiled4 256: WRONG"), "golden-model"),
    (TEXT_OUT.replace("sgemm 256: CORRECT\n", ""), "no sgemm verdict"),
    (TEXT_OUT.replace("sgemm 512x512x512: 0.049 ms/iter, 5478.2 GFLOPS\n", ""), "512"),
    (TEXT_OUT.replace("membw read (2048 MiB x4): 0.001 s, 6886.8 GB/s\n", ""), "membw"),
])
def test_text_rejections(out, msg):
    with pytest.raises(task_unit.UnitError, match=msg):
        task_unit.from_text(out)


def test_harness_failure_and_timeout(tmp_path):
    with pytest.raises(task_unit.UnitError, match="exited 1: CUDA error"):
        task_unit.run_unit(_home(tmp_path / "a", 'echo "CUDA error 100" >&2; exit 1\n'))
    with pytest.raises(task_unit.UnitError, match="timed out"):
        task_unit.run_unit(_home(tmp_path / "b", "sleep 5\n"), timeout=1)


def test_home_lookup(tmp_path, monkeypatch):
    monkeypatch.setattr(Path, "home", classmethod(lambda cls: tmp_path / "nohome"))
    monkeypatch.setattr(task_unit, "__file__", str(tmp_path / "pkg" / "task_unit.py"))
    monkeypatch.delenv("CLUSTER_GPU_HOME", raising=False)
    assert task_unit.gpu_home() is None
    with pytest.raises(task_unit.UnitError, match="no GPU home"):
        task_unit.run_unit()
    # the package layout: bin/gpu_workload + lib/switch_gpu.cubin
    pkg = tmp_path / "pkg"
    (pkg / "bin").mkdir(parents=True)
    (pkg / "lib").mkdir()
    exe = pkg / "bin" / "gpu_workload"
    exe.write_text("#!/bin/sh\n")
    exe.chmod(0o755)
    (pkg / "lib" / "switch_gpu.cubin").write_bytes(b"x")
    assert task_unit.gpu_home() == pkg
    # $CLUSTER_GPU_HOME comes first; a home without a module image does not qualify
    env_home = _home(tmp_path, "exit 0\n")
    monkeypatch.setenv("CLUSTER_GPU_HOME", str(env_home))
    assert task_unit.gpu_home() == env_home
    os.unlink(env_home / "switch_gpu_native.ptx")
    assert task_unit.gpu_home() == pkg


def test_verify_unit_rechecks():
    good = {"correct": True, "gflops": {"256": 1e3, "512": 5e3, "1024": 2e4}, "gbps": 6900.0}
    task_unit.verify_unit(good)
    for bad in ({**good, "correct": False}, {**good, "gbps": 9000.0}, {**good, "gflops": {"256": 1e3}}):
        with pytest.raises(task_unit.UnitError):
            task_unit.verify_unit(bad)


@pytest.mark.gpu
def test_unit_on_b200():
    """The real harness, built in this package, as one task unit."""
    r = task_unit.run_unit(PKG)
    assert r["correct"] is True and "B200" in r.get("device", "")
    assert {"sgemm", "sgemm_b200"} <= set(r["kernels_verified"])
    task_unit.verify_unit(r)
