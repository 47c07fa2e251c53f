"""Worker for the multi-GPU SGEMM test (run under torch.distributed.run,
one rank per GPU, NCCL): every rank computes its row panel with the CUDA
kernel, the panels are all-gathered -- by NCCL, or by the kernel itself
storing every tile into every rank's C over NVLink (gather_mode "peer",
run twice to cover the reuse of the mapped buffers) -- and each rank
checks the full C against the oracle on sampled rows plus a Freivalds check
of the whole product.  Exit status 0 = all ranks agree with the oracle."""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "switch-l4t-gpu_b200"))
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import orc  # noqa: E402
import sb200  # noqa: E402
import sgemm_dist  # noqa: E402


CASES = [(1000, 384, 1002, 1, "nccl"), (2048, 512, 256, 3, "nccl"), (257, 129, 67, 2, "nccl"),
         (1024, 512, 256, 1, "peer"), (2048, 1024, 512, 1, "peer"), (2048, 1024, 512, 1, "peer3x")]


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    sb200.init(local)
    bad = 0
    try:
        for ci, (M, N, K, chunks, mode) in enumerate(CASES):
            A = sb200.synth_uniform(M * K, -1.0, 1.0, 10 + ci).reshape(M, K)
            B = sb200.synth_uniform(K * N, -1.0, 1.0, 20 + ci).reshape(K, N)
            kern = "3xtf32" if mode == "peer3x" else "fp32"
            ps = sgemm_dist.PanelSgemm(M, N, K, chunks=chunks, gather_mode="nccl" if mode == "nccl" else "peer",
                                       kernel=kern)
            Ap = torch.from_numpy(A[ps.row0:ps.row1].copy()).to(dev)
            Bd = torch.from_numpy(B).to(dev)
            if mode != "nccl":
                ps.C.fill_(float("nan"))  # every cell must be written, by some rank
                torch.cuda.synchronize()
                dist.barrier()
                ps(Ap, Bd)
            C = ps(Ap, Bd).cpu().numpy()
            ps.close()
            rows = sorted(set([0, M - 1] + list(range(rank, M, max(1, M // 16)))))
            want = orc.sgemm(A, B)
            rel = np.linalg.norm(C[rows] - want[rows]) / np.linalg.norm(want[rows])
            fr = orc.freivalds(A, B, np.ascontiguousarray(C))
            ok = rel <= 1e-5 and fr <= 1e-5
            print(f"rank {rank} case {ci} M={M} N={N} K={K} chunks={chunks} {mode}: rel {rel:.2e} freivalds {fr:.2e} "
                  f"{'ok' if ok else 'BAD'}", flush=True)
            bad += 0 if ok else 1
        flag = torch.tensor([bad], device=dev)
        dist.all_reduce(flag)
        bad = int(flag.item())
    finally:
        dist.destroy_process_group()
    sys.exit(1 if bad else 0)


if __name__ == "__main__":
    main()
