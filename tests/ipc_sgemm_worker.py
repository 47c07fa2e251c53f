"""Child process of the CUDA IPC test: maps the C another process exported
(handle and offset on the command line) and stores the product A . B into
it and into a buffer of its own with sb_sgemm_multi, then unmaps it.  A and
B are regenerated from the same seeds as the parent's.  Prints the
checksum of its own copy; exit status 0 = the calls succeeded."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "switch-l4t-gpu_b200"))

import torch  # noqa: E402

import sb200  # noqa: E402


def main():
    handle, offset = bytes.fromhex(sys.argv[1]), int(sys.argv[2])
    M, N, K, seed = (int(v) for v in sys.argv[3:7])
    torch.cuda.set_device(0)
    torch.zeros(1, device="cuda")
    sb200.init(0)
    A = sb200.synth_uniform(M * K, -1.0, 1.0, seed).reshape(M, K)
    B = sb200.synth_uniform(K * N, -1.0, 1.0, seed + 1).reshape(K, N)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    peer = sb200.ipc_open(handle, offset)
    mine = torch.full((M, N), float("nan"), device="cuda")
    sb200.sgemm_multi(dA, dB, [mine, peer], M, N, K)
    torch.cuda.synchronize()
    sb200.ipc_close(peer, offset)
    print("checksum", float(mine.double().sum()), flush=True)


if __name__ == "__main__":
    main()
