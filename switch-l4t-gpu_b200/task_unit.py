"""Task-queue consumer of the SGEMM suite on a B200: run one unit of
`gpu_workload`, check its verdicts and numbers, return a small result dict.

The contract is the reference's deploy/cluster/gpu_task_example.py:
* GPU home: $CLUSTER_GPU_HOME, then ~/switch-l4t-gpu, then ~/gpu (:35-46).
  A home qualifies with an executable ./gpu_workload and a readable module
  image: the reference's ./switch_gpu_native.ptx, or this package's
  switch_gpu.cubin (flat, or under lib/ with the binary under bin/ -- the
  layout this package builds, which is also tried last).
* One unit: `gpu_workload --json <module>`; a harness that does not know
  --json is re-run in text mode (:110-116).
* JSON: `done` must be true, kernels.sgemm present and every verdict CORRECT,
  SGEMM timings for 256/512/1024 and membw_gbps present (:58-78).
* Text: the WORKLOAD_DONE sentinel, the verdict, timing and membw lines (:81-101).
* `verify_unit` re-checks a reported result on the coordinator (:129-133).

The sanity bounds are B200's, not the Tegra X1's (1000 GFLOPS and 1000 GB/s,
:22-23, which every B200 result exceeds): GFLOPS up to the FP32 FMA peak of
148 SMs x 128 lanes x 2 x 1.965 GHz = 74.4 TFLOP/s (the harness's own
fp32_peak_gflops_at_max_clock, when it reports one, is used instead), GB/s
up to HBM3e's nominal 8 TB/s.  A number above the physical peak is garbage,
not a fast GPU.  Errors are UnitError, as in the reference.
"""
import json
import os
import re
import subprocess
from pathlib import Path

SIZES = (256, 512, 1024)
TIMEOUT_S = 120  # first cuInit on a fresh node plus a 2 GiB bandwidth probe
GFLOPS_BOUNDS = (1.0, 74450.0)
GBPS_BOUNDS = (1.0, 8000.0)
PEAK_SLACK = 1.02  # event-timed SGEMM over the clock-derived peak: allowed margin

_RE_SGEMM_PERF = re.compile(r"^sgemm (\d+)x\1x\1: [\d.]+ ms/iter, ([\d.]+) GFLOPS", re.M)
_RE_MEMBW = re.compile(r"^membw read .* ([\d.]+) GB/s", re.M)
_RE_VERDICT = re.compile(r"^sgemm(?P<k>_\w+)? \d+: (?P<v>CORRECT|WRONG)\b", re.M)

MODULE_NAMES = ("switch_gpu_native.ptx", "switch_gpu.cubin")


class UnitError(ValueError):
    pass


def _harness_in(home):
    """(binary, module) of a qualifying home directory, else None."""
    layouts = [(home / "gpu_workload", [home / m for m in MODULE_NAMES]),
               (home / "bin" / "gpu_workload", [home / "lib" / "switch_gpu.cubin"])]
    for binary, modules in layouts:
        if binary.is_file() and os.access(binary, os.X_OK):
            for m in modules:
                if m.is_file() and os.access(m, os.R_OK):
                    return binary, m
    return None


def gpu_home():
    """Directory holding the harness and its module image, or None."""
    candidates = []
    if os.environ.get("CLUSTER_GPU_HOME"):
        candidates.append(Path(os.environ["CLUSTER_GPU_HOME"]))
    candidates += [Path.home() / "switch-l4t-gpu", Path.home() / "gpu", Path(__file__).resolve().parent]
    for c in candidates:
        if _harness_in(c):
            return c
    return None


def _check_numbers(gflops, gbps, peak=None):
    hi = GFLOPS_BOUNDS[1]
    if isinstance(peak, (int, float)) and peak > 0:
        hi = min(hi, peak * PEAK_SLACK)
    for s in map(str, SIZES):
        v = gflops.get(s)
        if not isinstance(v, (int, float)) or not GFLOPS_BOUNDS[0] <= v <= hi:
            raise UnitError(f"gflops[{s}] missing or outside sanity bounds")
    if not isinstance(gbps, (int, float)) or not GBPS_BOUNDS[0] <= gbps <= GBPS_BOUNDS[1]:
        raise UnitError("gbps missing or outside sanity bounds")


def _result(verified, gflops, gbps, peak=None, device=None):
    _check_numbers(gflops, gbps, peak)
    out = {"correct": True, "kernels_verified": sorted(verified),
           "gflops": {k: round(gflops[k], 1) for k in map(str, SIZES)}, "gbps": round(float(gbps), 1)}
    if device:
        out["device"] = device
    return out


def from_json(out):
    """Parse `gpu_workload --json` output; UnitError on any verdict or timing problem."""
    try:
        data = json.loads(out)
    except json.JSONDecodeError as exc:
        raise UnitError(f"invalid --json output: {exc}") from exc
    if data.get("done") is not True:
        raise UnitError("harness JSON truncated (done flag missing)")
    kernels = data.get("kernels")
    if not isinstance(kernels, dict) or not kernels.get("sgemm"):
        raise UnitError("harness JSON missing kernels.sgemm verdict")
    bad = sorted(k for k, v in kernels.items() if v != "CORRECT")
    if bad:
        raise UnitError(f"kernels failed the harness CPU golden-model check: {bad}")
    gflops = {}
    for r in data.get("sgemm") or []:
        if isinstance(r, dict) and isinstance(r.get("gflops"), (int, float)) and isinstance(r.get("n"), (int, float)):
            gflops[str(int(r["n"]))] = float(r["gflops"])
    missing = [s for s in map(str, SIZES) if s not in gflops]
    if missing:
        raise UnitError(f"no SGEMM timing for size(s) {missing}")
    return _result(kernels, gflops, data.get("membw_gbps"), data.get("fp32_peak_gflops_at_max_clock"),
                   data.get("device"))


def from_text(out):
    """Parse the human-readable lines of a harness run without --json."""
    if "WORKLOAD_DONE" not in out:
        raise UnitError("harness output truncated (no WORKLOAD_DONE sentinel)")
    verdicts = {"sgemm" + (m.group("k") or ""): m.group("v") for m in _RE_VERDICT.finditer(out)}
    if "sgemm" not in verdicts:
        raise UnitError("harness produced no sgemm verdict line")
    bad = sorted(k for k, v in verdicts.items() if v != "CORRECT")
    if bad:
        raise UnitError(f"kernels failed the harness CPU golden-model check: {bad}")
    gflops = {m.group(1): float(m.group(2)) for m in _RE_SGEMM_PERF.finditer(out)}
    missing = [s for s in map(str, SIZES) if s not in gflops]
    if missing:
        raise UnitError(f"no SGEMM timing for size(s) {missing}")
    mb = _RE_MEMBW.search(out)
    if mb is None:
        raise UnitError("harness produced no membw line")
    return _result(verdicts, gflops, float(mb.group(1)))


def run_unit(home=None, timeout=TIMEOUT_S):
    """One task unit: run the suite, return a small verifiable dict (or raise UnitError)."""
    home = Path(home) if home is not None else gpu_home()
    found = _harness_in(home) if home is not None else None
    if found is None:
        raise UnitError("no GPU home (CLUSTER_GPU_HOME / ~/switch-l4t-gpu / ~/gpu)")
    binary, module = map(str, found)
    try:
        proc = subprocess.run([binary, "--json", module], capture_output=True, text=True, timeout=timeout)
        if proc.returncode != 0 and not proc.stdout.lstrip().startswith("{"):
            # a harness without --json takes it for the module path: re-run in text mode
            proc = subprocess.run([binary, module], capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired as exc:
        raise UnitError(f"harness timed out after {timeout}s") from exc
    if proc.returncode != 0:
        raise UnitError(f"gpu_workload exited {proc.returncode}: {proc.stderr.strip()[:300]}")
    if proc.stdout.lstrip().startswith("{"):
        return from_json(proc.stdout)
    return from_text(proc.stdout)


def verify_unit(result):
    """Coordinator-side re-check of a reported result (UnitError rejects it)."""
    if result.get("correct") is not True:
        raise UnitError("result missing correct=true (golden-model check not reported)")
    _check_numbers(result.get("gflops", {}), result.get("gbps"))


if __name__ == "__main__":
    import sys
    try:
        print(json.dumps(run_unit(), indent=2))
    except UnitError as exc:
        sys.exit(f"unit failed: {exc}")
