"""Host logic of the row-panel sharded SGEMM on CPU ranks (gloo, world 2).

The CUDA product is replaced here by an exact stand-in (small-integer inputs,
so every ordering of the sums gives the same float) so that panel bounds,
padding of uneven M, the in-place all-gather and the chunked gather with its
final permutation are checked without a GPU.  The gathered C must equal the
oracle's restatement of the reference loop (gpu_workload.c:97-98) exactly.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sgemm_dist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exact_compute(A_panel, B, C_panel, rows, N, K, stream):
    C_panel.copy_((A_panel.double() @ B.double()).float())


def _operands(M, N, K, seed):
    g = np.random.default_rng(seed)
    A = g.integers(-8, 9, size=(M, K)).astype(np.float32)
    B = g.integers(-8, 9, size=(K, N)).astype(np.float32)
    return A, B


def _rank_main(rank, world, port, cases, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for ci, (M, N, K, chunks) in enumerate(cases):
            A, B = _operands(M, N, K, 100 + ci)
            ps = sgemm_dist.PanelSgemm(M, N, K, device="cpu", chunks=chunks, compute=_exact_compute)
            r0, r1 = sgemm_dist.panel_bounds(M, rank, world)
            assert (ps.row0, ps.row1) == (r0, r1)
            C = ps(torch.from_numpy(A[r0:r1].copy()), torch.from_numpy(B))
            np.save(os.path.join(outdir, f"c{ci}_r{rank}.npy"), C.numpy())
    finally:
        dist.destroy_process_group()


CASES = [(37, 20, 11, 1), (37, 20, 11, 3), (64, 16, 8, 2), (3, 5, 7, 1), (1, 4, 4, 1)]


@pytest.fixture(scope="module")
def gathered(tmp_path_factory):
    out = tmp_path_factory.mktemp("sgemm_dist")
    mp.start_processes(_rank_main, args=(2, _free_port(), CASES, str(out)), nprocs=2, start_method="spawn")
    return out


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_gathered_c_matches_oracle(gathered, ci):
    import orc
    M, N, K, _ = CASES[ci]
    A, B = _operands(M, N, K, 100 + ci)
    want = orc.sgemm(A, B)
    for rank in range(2):
        got = np.load(os.path.join(gathered, f"c{ci}_r{rank}.npy"))
        assert got.shape == (M, N)
        assert np.array_equal(got, want), f"rank {rank}"


def test_panel_bounds_cover_rows_once():
    for M in (1, 2, 7, 37, 16384):
        for world in (1, 2, 3, 4, 8):
            spans = [sgemm_dist.panel_bounds(M, r, world) for r in range(world)]
            rows = [i for a, b in spans for i in range(a, b)]
            assert rows == list(range(M))
            assert all(b - a <= sgemm_dist.panel_rows(M, world) for a, b in spans)


def test_rejects_bad_operands():
    ps = sgemm_dist.PanelSgemm(4, 4, 4, device="cpu", compute=_exact_compute)
    with pytest.raises(ValueError):
        ps(torch.zeros(3, 4), torch.zeros(4, 4))
    with pytest.raises(TypeError):
        ps(torch.zeros(4, 4, dtype=torch.float64), torch.zeros(4, 4, dtype=torch.float64))
