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


def _leaver_main(rank, world, port, outdir):
    """Rank 1 leaves after the first step (between steps, nothing in flight);
    rank 0's next gather must end with an error within the process group's
    short timeout instead of waiting for good."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    M, N, K = 16, 8, 4
    A, B = _operands(M, N, K, 7)
    ps = sgemm_dist.PanelSgemm(M, N, K, device="cpu", compute=_exact_compute)
    r0, r1 = sgemm_dist.panel_bounds(M, rank, world)
    Ap, Bt = torch.from_numpy(A[r0:r1].copy()), torch.from_numpy(B)
    ps(Ap, Bt)  # step 1: both ranks
    if rank == 1:
        os._exit(0)  # leaves without destroying the group
    t0 = time.time()
    try:
        ps(Ap, Bt)  # step 2: the peer is gone
        outcome = "no error"
    except Exception as ex:  # gloo reports the closed peer or the timeout
        outcome = "error: " + type(ex).__name__
    with open(os.path.join(outdir, "leaver.txt"), "w") as f:
        f.write(f"{outcome}\n{time.time() - t0:.2f}\n")
    os._exit(0)


def test_rank_leaving_between_steps_fails_fast(tmp_path):
    """Failure detection on the host: a rank that exits between steps makes
    the surviving rank's next all-gather raise within the process group's
    5 s timeout (plus slack), instead of hanging."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaver_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank was still waiting after 60 s"
    outcome, secs = (tmp_path / "leaver.txt").read_text().splitlines()[:2]
    assert outcome.startswith("error"), outcome
    assert float(secs) < 30.0


def test_rejects_bad_gather_mode():
    with pytest.raises(ValueError):
        sgemm_dist.PanelSgemm(4, 4, 4, device="cpu", compute=_exact_compute, gather_mode="bogus")


def _peer_on_cpu_main(rank, world, port, outdir):
    """The peer gather stores from this package's CUDA kernels into the
    other ranks' C; on CPU ranks (gloo) it must refuse at construction,
    before any collective, on every rank alike."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    outcome = "accepted"
    try:
        sgemm_dist.PanelSgemm(256, 128, 16, device="cpu", gather_mode="peer")
    except ValueError as ex:
        outcome = "ValueError: " + str(ex)
    with open(os.path.join(outdir, f"peer_cpu_{rank}.txt"), "w") as f:
        f.write(outcome + "\n")
    dist.destroy_process_group()


def test_peer_gather_refused_on_cpu_ranks(tmp_path):
    mp.start_processes(_peer_on_cpu_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        text = (tmp_path / f"peer_cpu_{r}.txt").read_text()
        assert text.startswith("ValueError") and "CUDA" in text, text
