"""SGEMM parity on the GPU: the drop-in kernels of switch_gpu.cubin launched
exactly as gpu_workload.c launches them, and the C-ABI sb_sgemm, against the
oracle's restatement of the harness's CPU triple loop (gpu_workload.c:97-98).

Tolerances: relative Frobenius error <= 1e-5 (the FP32 SGEMM bar), and zero
cells outside the harness's own |d| > 0.05|ref| + 1e-3 rule.  sgemm_naive
rounds like the CPU loop and must match it bit for bit."""
import numpy as np
import pytest

import drv
import orc
import sb200

pytestmark = pytest.mark.gpu
REL_FROB = 1e-5


def _mats(M, N, K, seed):
    A = sb200.synth_uniform(M * K, -1.0, 1.0, seed).reshape(M, K)
    B = sb200.synth_uniform(K * N, -1.0, 1.0, seed + 1).reshape(K, N)
    return A, B


def _rel_frob(C, ref):
    d = np.linalg.norm((C.astype(np.float64) - ref.astype(np.float64)).ravel())
    r = np.linalg.norm(ref.astype(np.float64).ravel())
    return d / max(r, 1e-30)


@pytest.fixture(scope="module")
def swmod(cuda_dev):
    return drv.Module(sb200.CUBINS["switch_gpu"])


@pytest.mark.parametrize("name,tile", [("sgemm_tiled", 32), ("sgemm_tiled4", 64), ("sgemm_opt", 64)])
@pytest.mark.parametrize("n", [256, 512, 1024])
def test_dropin_stock_geometry(cuda_dev, swmod, name, tile, n):
    import torch
    A, B = _mats(n, n, n, 11 + n)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.full((n, n), float("nan"), device="cuda")
    swmod.launch(name, (n // tile, n // tile), (16, 16), dA, dB, dC, n, n, n)
    torch.cuda.synchronize()
    C = dC.cpu().numpy()
    ref = orc.sgemm(A, B)
    assert np.isfinite(C).all()
    assert _rel_frob(C, ref) <= REL_FROB
    assert orc.sgemm_bad_cells(C, ref) == 0


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (33, 70, 129)])
def test_naive_bit_exact(cuda_dev, swmod, M, N, K):
    import torch
    A, B = _mats(M, N, K, 5)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros((M, N), device="cuda")
    swmod.launch("sgemm_naive", ((N + 15) // 16, (M + 15) // 16), (16, 16), dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), orc.sgemm(A, B))


def test_config0_1024_seed0(cuda_dev):
    """1024^3, A, B uniform[-1,1] from seed 0, C zeroed."""
    import torch
    n = 1024
    A, B = _mats(n, n, n, 0)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros((n, n), device="cuda")
    sb200.sgemm(dA, dB, dC, n, n, n)
    torch.cuda.synchronize()
    C = dC.cpu().numpy()
    assert _rel_frob(C, orc.sgemm(A, B)) <= REL_FROB


@pytest.mark.parametrize("M,N,K", [(129, 257, 100), (1, 1000, 3), (1000, 1, 7), (300, 200, 1), (130, 131, 133),
                                   (128, 128, 16), (0, 5, 5), (5, 5, 0)])
def test_ragged_shapes(cuda_dev, M, N, K):
    import torch
    A, B = _mats(max(M, 1), max(N, 1), max(K, 1), 3)
    A, B = A[:M, :K].copy(), B[:K, :N].copy()
    dA = torch.from_numpy(A).cuda() if A.size else torch.zeros(1, device="cuda")
    dB = torch.from_numpy(B).cuda() if B.size else torch.zeros(1, device="cuda")
    dC = torch.full((max(M, 1), max(N, 1)), 7.0, device="cuda")
    sb200.sgemm(dA, dB, dC, M, N, K)
    torch.cuda.synchronize()
    C = dC.cpu().numpy()[:M, :N]
    ref = orc.sgemm(A, B) if M and N else np.zeros((M, N), np.float32)
    if M and N:
        assert np.allclose(C, ref, rtol=1e-5, atol=1e-5)


def test_large_rows_and_freivalds(cuda_dev):
    """4096^3: sampled rows against the oracle loop, plus an FP64 Freivalds
    check of the whole product (size-independent property)."""
    import torch
    n = 4096
    A, B = _mats(n, n, n, 4096)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros((n, n), device="cuda")
    sb200.sgemm(dA, dB, dC, n, n, n)
    torch.cuda.synchronize()
    C = dC.cpu().numpy()
    rows = [0, 1, 127, 128, 2047, 4095]
    for r in rows:
        ref = orc.sgemm(A, B, r, r + 1)[r]
        assert _rel_frob(C[r], ref) <= REL_FROB
    assert orc.freivalds(A, B, C) < 1e-5
    C[1000, 17] += 1.0  # a single wrong cell is visible to the check
    assert orc.freivalds(A, B, C) > 1e-5


def test_16384_sampled_rows_and_freivalds(cuda_dev):
    """The largest SGEMM config (16384^3, 3 GB of operands and result): the
    harness's triple loop on sampled rows, and an FP64 Freivalds check of
    the whole product, where the full CPU loop would take hours."""
    import torch
    n = 16384
    A, B = _mats(n, n, n, 16384)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dC = torch.zeros((n, n), device="cuda")
    sb200.sgemm(dA, dB, dC, n, n, n)
    torch.cuda.synchronize()
    del dA, dB
    C = dC.cpu().numpy()
    del dC
    for r in (0, 8191, 16383):
        ref = orc.sgemm(A, B, r, r + 1)[r]
        assert _rel_frob(C[r], ref) <= REL_FROB
    assert orc.freivalds(A, B, C) < 1e-5
    # one wrong cell is visible: |C| ~ 43 here and ||A.B.r|| ~ 7e5, so an
    # error of 100 in one cell moves the check to ~1.4e-4
    C[12345, 678] += 100.0
    assert orc.freivalds(A, B, C) > 1e-5


def test_row_panels_assemble(cuda_dev):
    """sb_sgemm_rows over 4 panels (the multi-GPU shard unit) equals one call."""
    import torch
    M, N, K = 1000, 384, 256
    A, B = _mats(M, N, K, 9)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    full = torch.zeros((M, N), device="cuda")
    panels = torch.zeros((M, N), device="cuda")
    sb200.sgemm(dA, dB, full, M, N, K)
    bounds = [0, 250, 500, 750, 1000]
    for a, b in zip(bounds[:-1], bounds[1:]):
        sb200.sgemm_rows(dA, dB, panels, M, N, K, a, b)
    torch.cuda.synchronize()
    assert torch.equal(full, panels)


def test_membw_read4_checksum(cuda_dev, swmod):
    """membw_read4 semantics (switch_gpu.cu:41-54): out[i] = sum of thread i's
    float4s over `iters` passes; stock launch 512 x 256."""
    import torch
    n4 = 1 << 20
    buf = torch.rand(n4 * 4, device="cuda")
    out = torch.zeros(512 * 256, device="cuda")
    swmod.launch("membw_read4", (512,), (256,), buf, out, n4, 3)
    torch.cuda.synchronize()
    b = buf.view(-1, 4).sum(1).double().view(-1, 512 * 256)  # rows = strided passes
    ref = 3 * b.sum(0)
    assert torch.allclose(out.double(), ref, rtol=1e-5)


@pytest.mark.parametrize("M,N,K,row0,row1", [(1024, 1024, 2048, 256, 512), (256, 512, 4096, 0, 256),
                                             (1024, 1024, 1024, 0, 1024), (2048, 2048, 64, 0, 2048),
                                             (1152, 1152, 512, 0, 1152), (128, 128, 16, 0, 128)])
def test_split_k_small_products(cuda_dev, M, N, K, row0, row1):
    """Products with fewer 128x128 tiles than two per SM run stream-K (equal
    ranges of the tiles' k-chunks per CTA) and add each tile's pieces in CTA
    order: within the FP32 bar of the harness loop, and bit-identical from
    call to call (deterministic).  The cases cover ranges that span two
    tiles, ranges shorter than one chunk's worth per CTA (K = 64 over 256
    tiles) and a single whole tile."""
    import torch
    A, B = _mats(M, N, K, 77)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    outs = []
    for _ in range(2):
        dC = torch.full((M, N), 3.0, device="cuda")
        sb200.sgemm_rows(dA, dB, dC, M, N, K, row0, row1)
        torch.cuda.synchronize()
        outs.append(dC.cpu().numpy())
    C = outs[0]
    assert np.array_equal(outs[0], outs[1])
    assert _rel_frob(C[row0:row1], orc.sgemm(A, B, row0, row1)[row0:row1]) <= REL_FROB
    assert np.all(C[:row0] == 3.0) and np.all(C[row1:] == 3.0)  # rows outside the panel untouched


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (1000, 384, 1004), (129, 260, 36), (3, 4, 4),
                                   (1024, 1024, 1024), (128, 128, 32), (1152, 1152, 512)])
def test_sgemm_tma_bit_identical(cuda_dev, swmod, M, N, K):
    """The TMA-staged SGEMM gives the same bits as the register-staged kernel
    sgemm_b200 launched one CTA per tile (every output one fma chain over k
    in order) and meets the FP32 bar against the harness loop on sampled
    rows, ragged shapes included (TMA zero-fills outside the matrices).
    Products with fewer tiles than SMs (M, N % 128 == 0, K % 32 == 0) run
    stream-K -- each tile's k-slices split over CTAs, pieces added in CTA
    order -- so there the bar is the FP32 one on every row, and two calls
    give the same bits."""
    import torch
    A, B = _mats(M, N, K, 31)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    want = torch.zeros((M, N), device="cuda")
    got = torch.full((M, N), float("nan"), device="cuda")
    tiles = ((M + 127) // 128) * ((N + 127) // 128)
    swmod.launch("sgemm_b200", (tiles,), (256,), dA, dB, want, M, N, K)
    sb200.sgemm_tma(dA, dB, got, M, N, K)
    torch.cuda.synchronize()
    assert sb200.tc_error() == 0
    C = got.cpu().numpy()
    stream_k = tiles < sb200.sm_count() and M % 128 == 0 and N % 128 == 0 and K % 32 == 0
    if not stream_k:
        assert torch.equal(got, want)
        for r in sorted({0, M // 2, M - 1}):
            assert _rel_frob(C[r], orc.sgemm(A, B, r, r + 1)[r]) <= REL_FROB
    else:
        assert _rel_frob(C, orc.sgemm(A, B)) <= REL_FROB
        again = torch.full((M, N), float("nan"), device="cuda")
        sb200.sgemm_tma(dA, dB, again, M, N, K)
        torch.cuda.synchronize()
        assert torch.equal(got, again)


@pytest.mark.parametrize("M,N,K,nout", [(1024, 1024, 1024, 2), (256, 384, 48, 3), (128, 128, 16, 1)])
def test_sgemm_multi_outputs_bit_identical(cuda_dev, swmod, M, N, K, nout):
    """sb_sgemm_multi stores every tile into each output (here all on this
    GPU): each equals the one-CTA-per-tile sgemm_b200 launch bit for bit and
    meets the FP32 bar against the harness loop on sampled rows."""
    import torch
    A, B = _mats(M, N, K, 41)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    want = torch.zeros((M, N), device="cuda")
    swmod.launch("sgemm_b200", ((M // 128) * (N // 128),), (256,), dA, dB, want, M, N, K)
    outs = [torch.full((M, N), float("nan"), device="cuda") for _ in range(nout)]
    sb200.sgemm_multi(dA, dB, outs, M, N, K)
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, want)
    C = outs[0].cpu().numpy()
    for r in sorted({0, M // 2, M - 1}):
        assert _rel_frob(C[r], orc.sgemm(A, B, r, r + 1)[r]) <= REL_FROB


def test_sgemm_multi_rejects_partial_tiles(cuda_dev):
    import torch
    a = torch.zeros(256 * 64, device="cuda")
    for (M, N, K, nout) in [(100, 128, 16, 1), (128, 100, 16, 1), (128, 128, 20, 1), (128, 128, 16, 9)]:
        with pytest.raises(RuntimeError):
            sb200.sgemm_multi(a, a, [a] * nout, M, N, K)
