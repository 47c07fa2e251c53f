#!/usr/bin/env python3
"""bench.py -- headline benchmark of the B200 matrix-multiply hot path.

Workload: Qwen2.5-0.5B-architecture FP16-weight decode,
FP32 accumulate, random-init weights in the reference's file layout, 32
seeded prompt tokens, 256 new tokens, batch 1, KV cache up to 2048.  One
step = one generation request: prime the prompt, then decode 256 tokens.

  value   decode tokens/s over all ranks (the reference's own metric:
          generated tokens / generation-loop time, qwen_engine.c:549-551),
          CUDA events on the engine stream around the 256 decode steps,
          inputs resident, max over ranks.
  e2e     the same metric through the public C-ABI call with host buffers:
          sb_engine_generate (prompt ids in from pinned host memory,
          generated ids out), whole call timed per step.
  roofline  the dominant kernel of the step, timed standalone after an L2
          flush, algorithmic bytes / time vs the measured HBM copy peak.

N > 1 (torchrun): one independent replica per GPU (decode does not shard);
scaling "weak".  The weights (988 MB) exceed the 126 MB L2, so no flush is
needed between timed steps.

Secondary keys of the same line: "sgemm" -- 16384^3 FP32 SGEMM sharded by
row panels over all ranks (strong scaling), C gathered on every rank by the
kernel's own stores into the peers' C over NVLink (the NCCL all-gather of C
timed beside it), compute-only and with the gather, per-GPU fraction of the
live FP32 FMA peak; "sgemm_3xtf32" -- the same on the opt-in 3xTF32 tensor-core kernel;
"gemv" -- the standalone FP16 GEMV sweep (batch 1 on CUDA cores, 4 and 16
on the tcgen05 tensor cores) in GB/s against the HBM peak; "gpt2_decode" --
configs[1], GPT-2-124M-shape FP32 decode (16 prompt tokens, 128 new), with
its own e2e, roofline and reference CPU baseline; "sgemm_1024" -- configs[0]
(1024^3) beside the harness's CPU triple loop, and the CPU cpu_gemv_h per
GEMV shape under "gemv" (rank 0, N = 1).

`--impl reference` times the reference's own CPU decode (cpu_forward of
gpu-llm/engine/qwen_engine.c compiled unmodified into oracle/_ref) on the
host cores, one forked replica per core, on the same metric.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "switch-l4t-gpu_b200")
sys.path.insert(0, PKG)

N_PROMPT, N_GEN, MAX_CTX = 32, 256, 2048
WEIGHT_SEED = 20261201
METRIC = "Qwen-0.5B-shape FP16 decode tok/s"
UNIT = "tok/s"
BASELINE_TOKS = 8.9  # the reference's published Qwen2.5-0.5B FP16 decode rate on Tegra X1 (gpu-llm/STATUS.md:112)
FALLBACK_HBM_GBS = 6650.0
CPU_SAMPLE_TOKENS = 16  # per host core: about 10 s of reference CPU decode
CONFIG = {
    "workload": "qwen2.5-0.5b-fp16-decode (configs[2])",
    "arch": "Qwen2.5-0.5B: 24 layers, hidden 896, 14q/2kv heads x 64, SwiGLU 4864, vocab 151936 tied",
    "n_prompt": N_PROMPT, "n_gen": N_GEN, "batch": 1, "max_ctx": MAX_CTX,
    "weights": "random-init N(0,0.02) fp16 in the reference file layout (990,162,688 B)",
    "l2": "no flush: 988 MB of weights streamed per token > 126 MB L2",
}


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


RANK, WORLD, LOCAL_RANK = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def weights_path():
    d = "/dev/shm/sb200_bench" if os.path.isdir("/dev/shm") else "/tmp/sb200_bench"
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, f"qwen_{WEIGHT_SEED}.bin")


QWEN_FILE_BYTES = 990162688  # the reference's Qwen weight-file size (qwen_engine.c:61-75)
QWEN_V = 151936


def synth_tool():
    """The stand-alone synthetic-input writer (bin/sb_synth: sb_synth.c only,
    no CUDA and no libswitch_b200.so), so the reference arm never maps this
    package's GPU library."""
    exe = os.path.join(PKG, "bin", "sb_synth")
    if not os.access(exe, os.X_OK):
        raise RuntimeError("switch-l4t-gpu_b200/bin/sb_synth is not built (run __graft_entry__.build())")
    return exe


def ensure_weights(barrier):
    path = weights_path()
    if LOCAL_RANK == 0 and not (os.path.exists(path) and os.path.getsize(path) == QWEN_FILE_BYTES):
        tmp = path + f".tmp{os.getpid()}"
        subprocess.run([synth_tool(), "weights", "qwen", tmp, str(WEIGHT_SEED)], check=True, stdout=subprocess.DEVNULL)
        os.replace(tmp, path)
    barrier()
    return path


def prompt_ids(seed, n=N_PROMPT, vocab=QWEN_V):
    """The benchmark prompt (sb_synth_ids of `seed`), via bin/sb_synth."""
    out = subprocess.run([synth_tool(), "ids", str(n), str(vocab), str(seed)], check=True, capture_output=True,
                         text=True).stdout.split()
    return [int(v) for v in out]


def prompt_file(seed):
    path = os.path.join(os.path.dirname(weights_path()), f"prompt_{seed}_{N_PROMPT}.txt")
    with open(path, "w") as f:
        f.write("\n".join(str(i) for i in prompt_ids(seed)) + "\n")
    return path


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_index():
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ent = vis.split(",")
        if LOCAL_RANK < len(ent) and ent[LOCAL_RANK].strip().isdigit():
            return int(ent[LOCAL_RANK])
    return LOCAL_RANK


def ncu_traffic():
    """Per-launch DRAM bytes of the step kernels from the committed ncu summary."""
    p = os.path.join(REPO, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            return {k: v for k, v in json.load(f).items() if not k.startswith("_")}
    except (OSError, ValueError):
        return {}


# ------------------------------------------------------------------ CPU legs
def ref_bench_exe():
    exe = os.path.join(REPO, "oracle", "_ref", "ref_qwen_bench")
    return exe if os.access(exe, os.X_OK) else None


def run_ref_bench(path, procs, warmup, steps, tokens, prompt=None):
    exe = ref_bench_exe()
    cmd = [exe, path, str(procs), str(warmup), str(steps), str(tokens), "42"] + ([prompt] if prompt else [])
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    if out.returncode != 0:
        raise RuntimeError(f"ref_qwen_bench failed: {out.stderr[-400:]}")
    return json.loads(out.stdout.strip().splitlines()[-1])


PROMPT_SEED = 1000  # rank r of the GPU arm uses PROMPT_SEED + r; the CPU legs use rank 0's prompt


def cpu_baseline(path):
    """Reference CPU decode on this host's cores, bounded sample (rank 0, N=1):
    the same 32-token prompt primed untimed, then decode from position 32 on,
    as the GPU arm does."""
    cores = host_cores()
    if ref_bench_exe():
        r = run_ref_bench(path, cores, 0, 1, CPU_SAMPLE_TOKENS, prompt_file(PROMPT_SEED))
        return {"value": round(r["tok_s"], 4), "unit": UNIT, "cores": cores, "kind": "reference",
                "sample": f"{cores} forked replicas of the reference cpu_forward (qwen_engine.c:292-358) + argmax: "
                          f"the {N_PROMPT}-token prompt primed untimed, then {CPU_SAMPLE_TOKENS} greedy decode "
                          f"tokens each from position {N_PROMPT}; {r['timed_s']:.1f} s timed"}
    # oracle restatement (row-parallel threads) when the reference build is absent
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import numpy as np
    import orc
    m = orc.Model("qwen", path, N_PROMPT + 8, QWEN_V)
    ids = prompt_ids(PROMPT_SEED)
    for p_, t in enumerate(ids):
        logits = m.forward(t, p_, p_ == len(ids) - 1, nthreads=cores)
    tok = int(np.argmax(logits))
    t0 = time.perf_counter()
    for p_ in range(N_PROMPT, N_PROMPT + 2):
        tok = int(np.argmax(m.forward(tok, p_, True, nthreads=cores)))
    dt = time.perf_counter() - t0
    m.close()
    return {"value": round(2 / dt, 4), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"oracle restatement of cpu_forward, rows split over threads: prompt primed, "
                      f"2 decode tokens from position {N_PROMPT}"}


def run_reference_arm(args):
    """The reference's own CPU decode (cpu_forward + argmax of qwen_engine.c,
    compiled unmodified into oracle/_ref/ref_qwen_bench) on this host's
    cores.  This process maps no library of this package: the weight file
    and prompt come from bin/sb_synth, a separate CUDA-free program."""
    if RANK != 0:
        return
    line = {"impl": "reference", "metric": METRIC, "unit": UNIT, "higher_is_better": True}
    if not ref_bench_exe():
        line["unavailable"] = "oracle/_ref/ref_qwen_bench not built (needs the reference sources at build time)"
        print(json.dumps(line))
        return
    path = ensure_weights(lambda: None)
    cores = host_cores()
    r = run_ref_bench(path, cores, args.warmup, args.steps, 2, prompt_file(PROMPT_SEED))
    step_ms = 1e3 * r["timed_s"] / r["steps"]
    line.update({
        "value": round(r["tok_s"], 4), "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 3), "scaling": "weak", "vs_baseline": None, "dtype": "f16w-f32",
        "data": "synthetic",
        "config": dict(CONFIG, global_batch=WORLD, seq_len=N_PROMPT + N_GEN,
                       parallelism=f"replicas x{WORLD} (decode does not shard)"),
        "cpu_baseline": {"value": round(r["tok_s"], 4), "unit": UNIT, "cores": cores, "kind": "reference",
                         "sample": f"per step: {cores} forked replicas x 2 greedy decode tokens of the reference "
                                   f"cpu_forward, positions {N_PROMPT}+ after the same {N_PROMPT}-token prompt "
                                   f"(primed untimed) as the GPU arm"},
        "e2e": {"value": round(r["tok_s"], 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })
    print(json.dumps(line))


# ------------------------------------------------------------------ secondary GPU measurements
SGEMM_N = 16384
GEMV_SHAPES = [(896, 896), (4864, 896), (896, 4864), (151936, 896), (32768, 8192)]
L2_BYTES = 126e6  # B200 L2


def fp32_peak_tflops(torch, dev):
    """Live FP32 FMA throughput of this GPU (fma_peak kernel, CUDA events)."""
    import sb200
    out = torch.empty(8 * sb200.sm_count() * 256, dtype=torch.float32, device=dev)  # grid 8 x SMs of 256
    sb200.fma_peak(out, 2000)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    flops = sb200.fma_peak(out, 20000)
    e1.record()
    e1.synchronize()
    return flops / (e0.elapsed_time(e1) * 1e-3) / 1e12


def gathered_c_check(torch, dev, ps, B, n, dist_on):
    """Verify the all-gathered C on this rank without any CPU oracle: FP64
    Freivalds (C r against A (B r) for the WHOLE matrix, every rank's panel
    of A regenerated from its seed) and exact FP64 rows (4 per panel)
    against the harness rule |c - ref| <= 0.05 |ref| + 1e-3
    (gpu_workload.c:99-101).  Returns (freivalds rel err, sampled-row rel
    err, cells outside the rule), each the max over ranks."""
    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    r = torch.rand(n, generator=g, device=dev, dtype=torch.float64) * 2 - 1
    Bd = B.double()
    Br = Bd @ r
    lhs = ps.C.double() @ r
    rhs = torch.empty(n, dtype=torch.float64, device=dev)
    rows, idx = [], []
    for q in range(ps.world):
        r0, r1 = sgemm_dist_bounds(n, q, ps.world)
        gq = torch.Generator(device=dev)
        gq.manual_seed(5000 + q)
        Aq = torch.rand(r1 - r0, n, generator=gq, device=dev) * 2 - 1
        rhs[r0:r1] = Aq.double() @ Br
        pick = [0, (r1 - r0) // 3, 2 * (r1 - r0) // 3, r1 - r0 - 1]
        rows.append(Aq[pick].double())
        idx += [r0 + k for k in pick]
        del Aq
    fr = float(torch.linalg.norm(lhs - rhs) / torch.linalg.norm(rhs))
    want = torch.cat(rows) @ Bd
    got = ps.C[idx].double()
    rel = float(torch.linalg.norm(got - want) / torch.linalg.norm(want))
    bad = float(((got - want).abs() > 0.05 * want.abs() + 1e-3).sum())
    t = torch.tensor([fr, rel, bad], dtype=torch.float64, device=dev)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    del Bd, Br, lhs, rhs, want, got
    return float(t[0]), float(t[1]), int(t[2])


def sgemm_dist_bounds(M, rank, world):
    import sgemm_dist
    return sgemm_dist.panel_bounds(M, rank, world)


def sgemm_section(torch, dev, dist_on, steps, warmup, kernel="fp32"):
    """16384^3 FP32 SGEMM row-panel sharded over all ranks (strong scaling):
    compute-only and with the NCCL all-gather of C, max over ranks; at N > 1
    also the chunked form (4 row chunks, each gathered while the next is
    multiplied) and the fused form (the kernel stores every tile into every
    rank's C over NVLink: PanelSgemm gather_mode "peer"); the faster of the
    fused and the NCCL form is the reported path, and the C every rank holds
    after each is checked on every rank.
    kernel "3xtf32" is the opt-in tensor-pipe variant (reported separately)."""
    import sgemm_dist
    n = SGEMM_N
    ps = sgemm_dist.PanelSgemm(n, n, n, kernel=kernel)
    gA = torch.Generator(device=dev)
    gA.manual_seed(5000 + RANK)
    gB = torch.Generator(device=dev)
    gB.manual_seed(777)  # B is the same on every rank
    A = torch.rand(ps.rows, n, generator=gA, device=dev) * 2 - 1
    B = torch.rand(n, n, generator=gB, device=dev) * 2 - 1
    if kernel == "fp32":
        peak, peak_src, bound = fp32_peak_tflops(torch, dev), "fma_peak kernel, this run (of measured)", "fp32"
    else:
        mp = measured_peaks()
        bf16 = float(mp["bf16_tflops"]) if mp and mp.get("bf16_tflops") else 1590.0
        peak = bf16 / 2 / 3  # dense TF32 = half the bf16 rate; 3 products per useful one
        peak_src = ("measured bf16 cuBLAS / 2 (TF32) / 3 (products)" if mp and mp.get("bf16_tflops")
                    else "fallback 1590 bf16 / 2 / 3")
        bound = "tensor"
    cur = torch.cuda.current_stream(dev)

    def step():
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(cur)
        ps.multiply(A, B)
        e1.record(cur)
        if ps.world > 1:  # the gather PanelSgemm.__call__ issues after the product
            torch.distributed.all_gather_into_tensor(ps.C_pad, ps.C_pad[ps.rank * ps.R:(ps.rank + 1) * ps.R])
        e2.record(cur)
        return e0, e1, e2

    # the fused form (every tile stored into every rank's C by the kernel)
    # alternates with the NCCL form step by step, so both see the same
    # clocks and temperature (the 16384^3 products run at the power cap)
    pp = sgemm_dist.PanelSgemm(n, n, n, kernel=kernel, gather_mode="peer") if ps.world > 1 else None

    def peer_step():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        pp(A, B)
        e1.record(cur)
        return e0, e1

    for _ in range(max(1, warmup)):
        step()
        if pp is not None:
            peer_step()
    torch.cuda.synchronize()
    evs, pevs = [], []
    for _ in range(steps):
        evs.append(step())
        if pp is not None:
            pevs.append(peer_step())
    torch.cuda.synchronize()
    comp = sum(a.elapsed_time(b) for a, b, _ in evs)
    tot = sum(a.elapsed_time(c) for a, _, c in evs)
    peer_ms = sum(a.elapsed_time(b) for a, b in pevs)
    ov = 0.0
    if ps.world > 1:  # chunked: the gather of chunk i overlaps the product of chunk i + 1
        pc = sgemm_dist.PanelSgemm(n, n, n, kernel=kernel, chunks=4)
        for _ in range(max(1, warmup)):
            pc(A, B)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        for _ in range(steps):
            pc(A, B)
        e1.record(cur)
        torch.cuda.synchronize()
        ov = e0.elapsed_time(e1)
        del pc
        torch.cuda.empty_cache()
    t = torch.tensor([comp, tot, ov, peer_ms], dtype=torch.float64, device=dev)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    comp_ms, tot_ms, ov_ms, peer_ms = (float(v) / steps for v in t)
    # the C every rank holds after each gather form, checked on every rank
    checks = []
    for form in ([pp] if pp is not None else []) + [ps]:
        form(A, B)
        torch.cuda.synchronize()
        checks.append(gathered_c_check(torch, dev, form, B, n, dist_on))
    if pp is not None:
        pp.close()
        del pp
    fr, rel, bad = (max(c[i] for c in checks) for i in range(3))
    verdict = "CORRECT" if fr <= 1e-5 and rel <= 1e-5 and bad == 0 else "WRONG"
    flop = 2.0 * n ** 3
    per_gpu = 2.0 * ps.rows * n * n / (comp_ms * 1e-3) / 1e12
    # the faster of the two gather forms is the reported path; both times stay in the line
    fused = bool(peer_ms) and peer_ms <= tot_ms
    step_ms = peer_ms if fused else tot_ms
    res = {"n": n, "n_gpus": WORLD, "kernel": "sgemm_b200" if kernel == "fp32" else "sgemm_3xtf32_tc",
           "value": round(flop / (step_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "gather": ("tiles stored into every rank's C by the kernel (NVLink peer stores)" if fused
                      else "NCCL all-gather" if WORLD > 1 else "none (1 GPU)"),
           "compute_tflops": round(flop / (comp_ms * 1e-3) / 1e12, 2), "compute_ms": round(comp_ms, 3),
           "ms_per_step": round(step_ms, 3), "allgather_ms": round(tot_ms - comp_ms, 3)}
    if peer_ms:
        res["nccl_ms"] = round(tot_ms, 3)  # the panel, then the NCCL all-gather
        res["peer_ms"] = round(peer_ms, 3)  # the kernel's own stores into every rank's C
    if ov_ms:
        res["chunked4_ms"] = round(ov_ms, 3)
    res.update({"check": {"verdict": verdict, "freivalds": float("%.2e" % fr), "rows_rel": float("%.2e" % rel),
                          "bad_cells": bad},
                "roofline": {"bound": bound, "achieved_per_gpu": round(per_gpu, 2), "peak": round(peak, 2),
                             "frac": round(per_gpu / peak, 4), "peak_src": peak_src}})
    del A, B, ps
    torch.cuda.empty_cache()
    return res


GPT2_SEED, GPT2_PROMPT, GPT2_GEN, GPT2_CTX = 20261202, 16, 128, 1024
GPT2_CPU_TOKENS = 48  # per host core: about 10 s of reference CPU decode


def gpt2_section(torch, dev, dist, steps, warmup, with_cpu):
    """GPT-2-124M-shape FP32 greedy decode, 16 seeded
    prompt tokens, 128 new tokens, batch 1 -- the same measurements as the
    headline (resident decode, e2e through sb_engine_generate, roofline of
    the step kernel, reference CPU decode on the host cores)."""
    import ctypes
    import sb200

    def barrier():
        if dist:
            import torch.distributed as tdist
            tdist.barrier()

    d = os.path.dirname(weights_path())
    path = os.path.join(d, f"gpt2_{GPT2_SEED}.bin")
    if LOCAL_RANK == 0 and not (os.path.exists(path) and os.path.getsize(path) == sb200.GPT2["TOTAL_FLOATS"] * 4):
        tmp = path + f".tmp{os.getpid()}"
        sb200.synth_weights(sb200.MODEL_GPT2, tmp, GPT2_SEED)
        os.replace(tmp, path)
    barrier()
    V = sb200.GPT2["V"]
    eng = sb200.Engine(sb200.MODEL_GPT2, path, GPT2_CTX)
    ext = torch.cuda.ExternalStream(eng.stream, device=dev)
    prompt = sb200.synth_ids(GPT2_PROMPT, V, 2000 + RANK)

    def decode_step():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        eng.begin(prompt, GPT2_GEN)
        eng.steps(GPT2_PROMPT - 1, False)
        eng.steps(1, True)
        e0.record(ext)
        eng.steps(GPT2_GEN, True)
        e1.record(ext)
        ids = eng.finish(GPT2_PROMPT + GPT2_GEN + 1)
        assert len(ids) == GPT2_PROMPT + GPT2_GEN + 1
        return e0.elapsed_time(e1)

    pin_in = torch.tensor(prompt, dtype=torch.int32).pin_memory()
    pin_out = torch.zeros(GPT2_PROMPT + GPT2_GEN + 1, dtype=torch.int32).pin_memory()
    L = sb200.lib()
    nout = ctypes.c_int()

    def e2e_step():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        sb200.check(L.sb_engine_generate(eng.h, ctypes.c_void_p(pin_in.data_ptr()), GPT2_PROMPT, GPT2_GEN,
                                         ctypes.c_void_p(pin_out.data_ptr()), ctypes.byref(nout), 0))
        e1.record(ext)
        e1.synchronize()
        return e0.elapsed_time(e1)

    for _ in range(warmup):
        decode_step()
    torch.cuda.synchronize()
    barrier()
    ms = [decode_step() for _ in range(steps)]
    for _ in range(max(1, warmup // 2)):
        e2e_step()
    barrier()
    e2e_ms = [e2e_step() for _ in range(steps)]
    tot = torch.tensor([sum(ms), sum(e2e_ms)], dtype=torch.float64, device=dev)
    if dist:
        import torch.distributed as tdist
        tdist.all_reduce(tot, op=tdist.ReduceOp.MAX)
    total_ms, e2e_total = float(tot[0].item()), float(tot[1].item())
    value = WORLD * steps * GPT2_GEN / (total_ms / 1e3)
    peaks = measured_peaks()
    peak = float(peaks["hbm_gbs"]) if peaks and peaks.get("hbm_gbs") else FALLBACK_HBM_GBS
    tok_ms = total_ms / (steps * GPT2_GEN)
    step_bytes = eng.step_bytes()
    achieved = step_bytes / (tok_ms * 1e-3) / 1e9
    dom = eng.step_kernel
    out = {
        "metric": "GPT-2-124M-shape FP32 decode tok/s", "value": round(value, 2), "unit": UNIT,
        "ms_per_step": round(total_ms / steps, 3), "steps": steps, "dtype": "f32",
        "config": {"workload": "gpt2-124m-fp32-decode (configs[1])", "n_prompt": GPT2_PROMPT, "n_gen": GPT2_GEN,
                   "batch": 1, "max_ctx": GPT2_CTX,
                   "weights": "random-init N(0,0.02) fp32 in the reference file layout (497,759,232 B)"},
        "e2e": {"value": round(WORLD * steps * GPT2_GEN / (e2e_total / 1e3), 2), "unit": UNIT,
                "h2d_bytes_per_step": GPT2_PROMPT * 4 + 48, "d2h_bytes_per_step": (GPT2_PROMPT + GPT2_GEN + 1) * 4 + 48,
                "note": "sb_engine_generate: prompt from pinned host memory, batched 3xTF32 prefill of the first "
                        "15 prompt tokens, 129 decode steps, ids back"},
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": ncu_traffic().get("gpt2_decode_mk") if eng.persistent
                     else None, "bytes_per_launch": step_bytes, "launch_us": round(tok_ms * 1e3, 2)},
        "gpu_launches": steps * GPT2_GEN * eng.launches_per_step(True),
        "step_kernel": "persistent whole-step kernel (1 cooperative launch per token)" if eng.persistent
        else "one kernel per stage (63 launches per token)",
    }
    eng.close()
    exe = os.path.join(REPO, "oracle", "_ref", "ref_gpt2_bench")
    if with_cpu and RANK == 0 and WORLD == 1 and os.access(exe, os.X_OK):
        try:
            cores = host_cores()
            r = subprocess.run([exe, path, str(cores), "0", "1", str(GPT2_CPU_TOKENS), "42"],
                               capture_output=True, text=True, timeout=900)
            j = json.loads(r.stdout.strip().splitlines()[-1])
            out["cpu_baseline"] = {"value": round(j["tok_s"], 4), "unit": UNIT, "cores": cores, "kind": "reference",
                                   "sample": f"{cores} forked replicas of the reference cpu_forward "
                                             f"(gpt2_engine.c:363-421) + argmax, {GPT2_CPU_TOKENS} greedy decode "
                                             f"tokens each; {j['timed_s']:.1f} s wall"}
        except Exception as ex:  # reported, not fatal
            out["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
    return out


def gemv_section(torch, dev):
    """Standalone FP16 GEMV sweep y = W.x (fp16 W and x, fp32 y) at batch 1
    (CUDA cores), 4 and 16 (tcgen05 tensor cores); W copies rotated through
    1 GiB so every launch streams from HBM.  The timed launches are replayed
    from a CUDA graph, so the small shapes measure the kernels, not the
    per-call Python launch path."""
    import sb200
    peaks = measured_peaks()
    peak = float(peaks["hbm_gbs"]) if peaks and peaks.get("hbm_gbs") else FALLBACK_HBM_GBS
    pool = torch.empty(1 << 29, dtype=torch.float16, device=dev).normal_(0, 0.02)  # 1 GiB
    side = torch.cuda.Stream(dev)
    out = {}
    for (N, K) in GEMV_SHAPES:
        wsz = N * K
        # enough W copies to rotate through > 4 x the 126 MB L2, so no launch
        # finds its weights in L2 (the 1 GiB pool bounds the count)
        ncopy = max(1, min(pool.numel() // wsz, int(4 * L2_BYTES / (wsz * 2)) + 1))
        reps = max(8, min(400, int(4e9 / (wsz * 2))))
        for Bw in (1, 4, 16):
            X = torch.randn(Bw, K, device=dev).half()
            Y = torch.empty(Bw, N, device=dev)
            fn = sb200.gemv_hh if Bw == 1 else sb200.gemm_hh  # batches 4 and 16: tcgen05 tensor cores
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):  # warm-up (workspaces are allocated here, outside the capture)
                for i in range(min(ncopy, 4)):
                    fn(pool[i * wsz:(i + 1) * wsz], X, Y, K, N, Bw, stream=side)
            side.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                cap = torch.cuda.current_stream(dev)
                for r in range(reps):
                    i = r % ncopy
                    fn(pool[i * wsz:(i + 1) * wsz], X, Y, K, N, Bw, stream=cap)
            graph.replay()  # warm replay
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            del graph
            us = e0.elapsed_time(e1) * 1e3 / reps
            nbytes = wsz * 2 + Bw * K * 2 + Bw * N * 4
            gbs = nbytes / (us * 1e-6) / 1e9
            out[f"{N}x{K}_b{Bw}"] = {"us": round(us, 2), "GB/s": round(gbs, 1), "frac": round(gbs / peak, 4),
                                     "l2": "rotating copies" if ncopy * wsz * 2 > 4 * L2_BYTES else "L2-resident",
                                     "launches": "CUDA-graph replay of %d" % reps}
    del pool
    torch.cuda.empty_cache()
    return {"metric": "FP16 GEMV HBM GB/s", "kernel": "b1: gemv_hh1, or gemv_hh_sk1 (split-K) below 2 x SMs four-row tasks (CUDA cores); b4, b16: gemm_hh_tc (tcgen05), or gemm_hh_mma8/16 (mma.sync, one launch) below 2 x SMs eight-row tiles",
            "peak": peak, "unit": "GB/s", "shapes": out}


def cpu_paths_baseline(torch, dev):
    """configs[0] and configs[3] beside their reference CPU paths, timed on
    the host cores (rank 0, N = 1): the harness's SGEMM triple loop
    (gpu_workload.c:97-98) at 1024^3 and cpu_gemv_h (qwen_engine.c:276-284)
    per GEMV shape, each as the oracle's C restatement, on one thread and
    row-parallel over all cores (arithmetic unchanged)."""
    import ctypes
    import numpy as np
    import sb200
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import orc
    cores = host_cores()
    rng = np.random.default_rng(0)
    n = 1024
    A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    B = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    rows1 = 64  # single-thread sample: 1/16 of the rows
    t0 = time.perf_counter()
    orc.sgemm(A, B, 0, rows1, nthreads=1)
    g1 = 2.0 * rows1 * n * n / (time.perf_counter() - t0) / 1e9
    t0 = time.perf_counter()
    orc.sgemm(A, B, 0, n, nthreads=cores)
    gall = 2.0 * n ** 3 / (time.perf_counter() - t0) / 1e9
    dA, dB = torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev)
    dC = torch.empty(n, n, device=dev)
    for _ in range(5):
        sb200.sgemm(dA, dB, dC, n, n, n)
    # the 12 MB of operands fit in L2: write 256 MB before each launch and
    # time the launches one by one
    flush = torch.empty(1 << 26, dtype=torch.float32, device=dev)
    reps = 50
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        sb200.sgemm(dA, dB, dC, n, n, n)
        e1.record()
    torch.cuda.synchronize()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / reps
    del flush
    gpu_tf = 2.0 * n ** 3 / (ms * 1e-3) / 1e12
    out = {"sgemm_1024": {
        "metric": "SGEMM TFLOPS", "n": n, "value": round(gpu_tf, 2), "unit": "TFLOP/s",
        "config": "configs[0]: 1024^3 FP32, A and B U[-1,1] from seed 0; L2 flushed (256 MB written) before "
                  "each timed launch",
        "cpu_baseline": {"value": round(gall / 1e3, 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "gflops_1_thread": round(g1, 3), "gflops_all_cores": round(gall, 2),
                         "sample": f"oracle restatement of the harness triple loop: {rows1} rows on 1 thread, "
                                   f"all 1024 rows row-parallel on {cores} threads"}}}
    gem = {}
    L = orc.oracle()
    for (N, K) in GEMV_SHAPES:
        W = rng.normal(0, 0.02, (N, K)).astype(np.float16).view(np.uint16)
        x = rng.normal(0, 1, K).astype(np.float32)
        y = np.zeros(N, dtype=np.float32)
        res = {}
        for label, th in (("1_thread", 1), ("all_cores", cores)):
            t0 = time.perf_counter()
            L.orc_gemv_h(W.ctypes.data_as(ctypes.c_void_p), x.ctypes.data_as(ctypes.c_void_p), None,
                         y.ctypes.data_as(ctypes.c_void_p), K, N, th)
            dt = time.perf_counter() - t0
            res[f"GB/s_{label}"] = round((N * K * 2 + K * 4 + N * 4) / dt / 1e9, 2)
        gem[f"{N}x{K}_b1"] = res
    out["gemv_cpu"] = {"kind": "port", "cores": cores,
                       "sample": "oracle restatement of cpu_gemv_h (fp16 W, fp32 x), whole matrix per shape",
                       "shapes": gem}
    return out


# ------------------------------------------------------------------ GPU arm
def run_b200(args):
    import torch
    import sb200

    dist = WORLD > 1
    if dist:
        import datetime
        import torch.distributed as tdist
        torch.cuda.set_device(LOCAL_RANK)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", LOCAL_RANK))

        def barrier():
            tdist.barrier()
    else:
        def barrier():
            pass
    dev = torch.device("cuda", LOCAL_RANK)
    torch.cuda.set_device(dev)
    torch.zeros(1, device=dev)
    sb200.init(LOCAL_RANK)
    path = ensure_weights(barrier)

    eng = sb200.Engine(sb200.MODEL_QWEN, path, MAX_CTX)
    ext = torch.cuda.ExternalStream(eng.stream, device=dev)
    prompt = sb200.synth_ids(N_PROMPT, sb200.QWEN["V"], PROMPT_SEED + RANK)

    def decode_step():
        """One request with resident inputs: returns decode-loop ms (events)."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        eng.begin(prompt, N_GEN)
        eng.steps(N_PROMPT - 1, False)  # prompt tokens, no LM head
        eng.steps(1, True)  # last prompt token -> first generated token
        e0.record(ext)
        eng.steps(N_GEN, True)  # the 256 timed decode steps
        e1.record(ext)
        ids = eng.finish(N_PROMPT + N_GEN + 1)
        assert len(ids) == N_PROMPT + N_GEN + 1
        return e0.elapsed_time(e1)

    for _ in range(args.warmup):
        decode_step()
    torch.cuda.synchronize()
    barrier()
    clocks = Clocks(gpu_index())
    if RANK == 0:
        clocks.start()
        time.sleep(0.3)
    t_wall0 = time.perf_counter()
    ms = [decode_step() for _ in range(args.steps)]
    torch.cuda.synchronize()
    wall = time.perf_counter() - t_wall0
    clk = clocks.stop() if RANK == 0 else None
    barrier()
    total = torch.tensor([sum(ms)], dtype=torch.float64, device=dev)
    if dist:
        import torch.distributed as tdist
        tdist.all_reduce(total, op=tdist.ReduceOp.MAX)
    total_ms = float(total.item())
    value = WORLD * args.steps * N_GEN / (total_ms / 1e3)

    # ---- e2e through the public C-ABI call, host (pinned) buffers
    pin_in = torch.tensor(prompt, dtype=torch.int32).pin_memory()
    pin_out = torch.zeros(N_PROMPT + N_GEN + 1, dtype=torch.int32).pin_memory()
    import ctypes
    L = sb200.lib()
    nout = ctypes.c_int()

    def e2e_step():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        sb200.check(L.sb_engine_generate(eng.h, ctypes.c_void_p(pin_in.data_ptr()), N_PROMPT, N_GEN,
                                         ctypes.c_void_p(pin_out.data_ptr()), ctypes.byref(nout), 0))
        e1.record(ext)
        e1.synchronize()
        return e0.elapsed_time(e1)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    barrier()
    e2e_ms = [e2e_step() for _ in range(args.steps)]
    e2e_total = torch.tensor([sum(e2e_ms)], dtype=torch.float64, device=dev)
    if dist:
        import torch.distributed as tdist
        tdist.all_reduce(e2e_total, op=tdist.ReduceOp.MAX)
    e2e_value = WORLD * args.steps * N_GEN / (float(e2e_total.item()) / 1e3)

    # ---- roofline of the dominant kernel.  With the persistent whole-step
    # kernel (one launch per token) the dominant kernel IS the step: its
    # launch duration is the event-timed decode time per token, its
    # algorithmic bytes the step's weight bytes.  With one kernel per stage
    # the dominant stage kernel is timed standalone after an L2 flush.
    peaks = measured_peaks()
    peak = float(peaks["hbm_gbs"]) if peaks and peaks.get("hbm_gbs") else FALLBACK_HBM_GBS
    peak_src = "measured" if peaks and peaks.get("hbm_gbs") else "fallback"
    step_bytes = eng.step_bytes()
    tok_ms = total_ms / (args.steps * N_GEN)
    if eng.persistent:
        dom, dbytes, dms = eng.step_kernel, step_bytes, tok_ms
        kernels = {}
    else:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        prof = {}
        for name, kid, per_step in (("qwen_gateup_swiglu", eng.K_MLP_UP, 24), ("qwen_lmhead", eng.K_LMHEAD, 1),
                                    ("qwen_gemv_resid(down)", eng.K_MLP_DOWN, 24), ("qwen_qkv_rope", eng.K_QKV, 24),
                                    ("qwen_gemv_resid(o)", eng.K_O, 24)):
            kms, kbytes = eng.profile(kid, 20, flush, flush.numel())
            prof[name] = {"ms": kms, "bytes": kbytes, "per_step": per_step}
        del flush
        dom = max(prof, key=lambda k: prof[k]["ms"] * prof[k]["per_step"])
        dbytes, dms = prof[dom]["bytes"], prof[dom]["ms"]
        kernels = {k: {"GB/s": round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1), "us": round(v["ms"] * 1e3, 2)}
                   for k, v in prof.items()}
    achieved = dbytes / (dms * 1e-3) / 1e9
    traffic = ncu_traffic().get(dom)
    roofline = {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_src,
                "bytes_per_launch": dbytes, "launch_us": round(dms * 1e3, 2),
                "step_frac": round(step_bytes / (tok_ms * 1e-3) / 1e9 / peak, 4)}
    if kernels:
        roofline["kernels"] = kernels

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": WORLD, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / BASELINE_TOKS, 1), "dtype": "f16w-f32", "data": "synthetic",
        "config": dict(CONFIG, global_batch=WORLD, seq_len=N_PROMPT + N_GEN,
                       parallelism=f"replicas x{WORLD} (decode does not shard)"),
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": N_PROMPT * 4 + 48,
                "d2h_bytes_per_step": (N_PROMPT + N_GEN + 1) * 4 + 48,
                "note": "sb_engine_generate: prompt from pinned host memory, batched tensor-core prefill of "
                        "the first 31 prompt tokens, 257 decode steps, ids back"},
        "gpu_launches": args.steps * N_GEN * eng.launches_per_step(True),
        "step_kernel": "persistent whole-step kernel (1 cooperative launch per token)" if eng.persistent
        else "one kernel per stage (123 launches per token)",
        "roofline": roofline,
        "clocks": clk,
        "wall_s_timed": round(wall, 3),
    }
    eng.close()
    if not args.no_secondary:
        # the latency-bound sections first: the 16384^3 SGEMMs that follow
        # run at the power cap, and the GPU's clocks take a while to recover
        line["gemv"] = gemv_section(torch, dev)
        line["gpt2_decode"] = gpt2_section(torch, dev, dist, max(3, args.steps // 2), 3, not args.no_cpu_baseline)
        # measured here, printed last (see below)
        sg = sgemm_section(torch, dev, dist, max(3, args.steps // 2), 3)
        sg3 = sgemm_section(torch, dev, dist, max(3, args.steps // 2), 3, kernel="3xtf32")
    if RANK == 0 and WORLD == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline(path)
        except Exception as ex:  # reported, not fatal
            line["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
        if not args.no_secondary:
            try:
                extra = cpu_paths_baseline(torch, dev)
                line["sgemm_1024"] = extra["sgemm_1024"]
                line["gemv"]["cpu_baseline"] = extra["gemv_cpu"]
            except Exception as ex:  # reported, not fatal
                line["sgemm_1024"] = {"error": str(ex)[:200]}
    if not args.no_secondary:
        # the strong-scaling SGEMM rows of configs[4] close the line, so a
        # reader that keeps only its tail still has them at every N
        line["sgemm_note"] = ("configs[4]: 16384^3 FP32 row panels over n_gpus ranks, B replicated; C gathered "
                              "by peer stores from the kernel (peer_ms) or an NCCL all-gather (nccl_ms), the faster reported; value "
                              "includes the gather; per-GPU roofline vs the live FMA peak; gathered C checked on "
                              "every rank (FP64 Freivalds + exact rows)")
        line["sgemm"] = sg
        line["sgemm_3xtf32"] = sg3
    if RANK == 0:
        print(json.dumps(line, separators=(",", ":")))
    if dist:
        import torch.distributed as tdist
        barrier()
        tdist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the SGEMM and GEMV sweep measurements")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
