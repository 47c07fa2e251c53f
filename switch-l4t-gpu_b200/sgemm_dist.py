"""sgemm_dist.py -- row-panel sharded SGEMM over the ranks of one node.

C = A.B with A [M x K], B [K x N], C [M x N], FP32, row-major -- the
contract of the reference's sgemm kernels (switch_gpu.cu:5-39, launched by
gpu_workload.c:88-90) -- split across P ranks, one process per GPU:

  * rank p owns the row panel C[p*R : p*R + rows_p] (R = ceil(M/P)) and
    computes it from its rows of A and a replicated B with this package's
    sgemm_b200 kernel (sb_sgemm through the C-ABI); no data crosses NVLink
    during the product;
  * when the caller wants the full C on every rank, one NCCL all-gather of
    the panels follows on the same stream.  Row-major panels are contiguous,
    so the gather runs in place into a (P*R) x N buffer whose first M rows
    are C: no reshuffle.
  * chunks > 1 splits each panel into row chunks and gathers chunk i while
    chunk i+1 is multiplied (gather on a second stream, ordered by events);
    the chunk-major staging is permuted into C with one device copy at the
    end.
  * gather_mode="peer" fuses the gather into the product: every rank maps
    the other ranks' C into its process (CUDA IPC), and the kernel
    (sb_sgemm_multi) stores each finished 128 x 128 tile into all of them
    over NVLink while it multiplies the next -- no all-gather, no staging.
    One-element collectives before and after order it: nobody still reads
    the previous C when the stores start, and every rank's tiles have
    landed when the call's stream moves on.

The reference has no multi-GPU path; the sharding rule (row panels, B
replicated, all-gather of C) is this package's own.  The compute hook exists
so the host logic (bounds, padding, gather order) can be exercised on CPU
ranks in tests; the default -- and the only product path -- is the CUDA
kernel, which raises if the extension library cannot be loaded.
"""
import torch
import torch.distributed as dist


def panel_rows(M, world):
    """Rows per rank (the last panels may hold fewer real rows)."""
    return (M + world - 1) // world


def panel_bounds(M, rank, world):
    """[row0, row1) of C computed by `rank`."""
    rp = panel_rows(M, world)
    r0 = min(M, rank * rp)
    return r0, min(M, r0 + rp)


def _cuda_compute(A_panel, B, C_panel, rows, N, K, stream):
    import sb200
    sb200.sgemm(A_panel, B, C_panel, rows, N, K, stream)


def _tf32x3_compute(A_panel, B, C_panel, rows, N, K, stream):
    import sb200
    sb200.sgemm_3xtf32(A_panel, B, C_panel, rows, N, K, stream)


KERNELS = {"fp32": _cuda_compute, "3xtf32": _tf32x3_compute}


class PanelSgemm:
    """Reusable buffers for C = A.B sharded by row panels over `group`.

    A_panel: this rank's rows [row0, row1) of A (contiguous, rows x K).
    B:       the whole B (K x N), replicated on every rank.
    kernel:  "fp32" (CUDA-core FFMA, the default) or "3xtf32" (opt-in, the
             TF32 tensor pipe with the 3xTF32 split).
    gather_mode: "nccl" (the panel, then an NCCL all-gather) or "peer" (the
             kernel stores every tile into every rank's C; needs M a
             multiple of 128 x world, N of 128 and K of 16; call close()
             on every rank before the buffers go away).
    """

    def __init__(self, M, N, K, group=None, device=None, chunks=1, compute=None, kernel="fp32", gather_mode="nccl"):
        if M <= 0 or N <= 0 or K <= 0 or chunks < 1:
            raise ValueError("PanelSgemm: M, N, K and chunks must be positive")
        self.M, self.N, self.K = M, N, K
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.R = panel_rows(M, self.world)
        self.row0, self.row1 = panel_bounds(M, self.rank, self.world)
        self.rows = self.row1 - self.row0
        self.chunks = max(1, min(chunks, self.R))
        if kernel not in KERNELS:
            raise ValueError(f"PanelSgemm: kernel must be one of {sorted(KERNELS)}")
        self.compute = compute or KERNELS[kernel]
        # gathered C, padded to P*R rows; rows [0, M) are the product
        self.C_pad = torch.empty(self.world * self.R, N, dtype=torch.float32, device=self.device)
        self.C = self.C_pad[:M]
        if self.chunks > 1:
            self.rc = panel_rows(self.R, self.chunks)  # rows per chunk (padded)
            self.stage = torch.empty(self.chunks, self.world, self.rc, N, dtype=torch.float32, device=self.device)
            self.mine = torch.empty(self.chunks, self.rc, N, dtype=torch.float32, device=self.device)
        self.is_cuda = self.device.type == "cuda"
        self.comm = torch.cuda.Stream(self.device) if self.is_cuda and self.chunks > 1 else None
        if gather_mode not in ("nccl", "peer"):
            raise ValueError("PanelSgemm: gather_mode must be 'nccl' or 'peer'")
        self.gather_mode = gather_mode if self.world > 1 else "nccl"
        self._peers = {}
        if self.gather_mode == "peer":
            if compute is not None or self.chunks != 1 or not self.is_cuda:
                raise ValueError("PanelSgemm: peer gather runs this package's CUDA kernels, chunks=1")
            self._multi = "sgemm_multi" if kernel == "fp32" else "sgemm_3xtf32_multi"
            if M % (128 * self.world) or N % 128 or K % 16:
                raise ValueError("PanelSgemm: peer gather needs M % (128 x world) == 0, N % 128 == 0, K % 16 == 0")
            self._open_peers()

    def _open_peers(self):
        import sb200
        mine = sb200.ipc_export(self.C_pad)
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=self.group)
        base = {}
        for r in range(self.world):
            if r == self.rank:
                base[r] = self.C_pad.data_ptr()
            else:
                base[r] = sb200.ipc_open(*every[r])
                self._peers[r] = (base[r], every[r][1])
        # this rank's panel rows inside every rank's C; its own C first
        off = self.row0 * self.N * 4
        self._dsts = [base[self.rank] + off] + [base[r] + off for r in range(self.world) if r != self.rank]
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)

    def close(self):
        """Unmap the peers' C (peer gather; a collective: every rank calls it)."""
        if self.gather_mode != "peer" or not self._peers:
            return
        import sb200
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still stores into a C
        for addr, off in self._peers.values():
            sb200.ipc_close(addr, off)
        self._peers = {}
        dist.barrier(group=self.group)  # every mapping is gone before an owner may free its C

    def panel(self):
        """This rank's panel of C (a view of the gathered buffer)."""
        return self.C_pad[self.rank * self.R:self.rank * self.R + self.rows]

    def _check(self, A_panel, B):
        if tuple(A_panel.shape) != (self.rows, self.K) or tuple(B.shape) != (self.K, self.N):
            raise ValueError(f"PanelSgemm: A panel must be {self.rows}x{self.K} and B {self.K}x{self.N}")
        if A_panel.dtype != torch.float32 or B.dtype != torch.float32:
            raise TypeError("PanelSgemm: FP32 operands required")
        if not (A_panel.is_contiguous() and B.is_contiguous()):
            raise ValueError("PanelSgemm: contiguous row-major operands required")

    def _stream(self, stream):
        if not self.is_cuda:
            return None
        return stream if stream is not None else torch.cuda.current_stream(self.device)

    def multiply(self, A_panel, B, stream=None):
        """This rank's panel only (no communication), on `stream` (default:
        the current torch stream)."""
        self._check(A_panel, B)
        if self.rows:
            self.compute(A_panel, B, self.panel(), self.rows, self.N, self.K, self._stream(stream))
        return self.panel()

    def __call__(self, A_panel, B, gather=True, stream=None):
        """Panel product, then (gather=True) the full C on every rank."""
        if not gather or self.world == 1:
            self.multiply(A_panel, B, stream)
            return self.C if self.world == 1 else self.panel()
        if self.gather_mode == "peer":
            import sb200
            if not self._peers:
                raise RuntimeError("PanelSgemm: closed")
            self._check(A_panel, B)
            s = self._stream(stream)
            with torch.cuda.stream(s):
                dist.all_reduce(self._flag, op=dist.ReduceOp.MAX, group=self.group)  # the previous C is read
                getattr(sb200, self._multi)(A_panel, B, self._dsts, self.rows, self.N, self.K, s)
                dist.all_reduce(self._flag, op=dist.ReduceOp.MAX, group=self.group)  # every panel has landed
            return self.C
        if self.chunks == 1:
            s = self._stream(stream)
            self.multiply(A_panel, B, s)
            mine = self.C_pad[self.rank * self.R:(self.rank + 1) * self.R]
            if s is None:
                dist.all_gather_into_tensor(self.C_pad, mine, group=self.group)
            else:
                with torch.cuda.stream(s):  # the gather is ordered after the product
                    dist.all_gather_into_tensor(self.C_pad, mine, group=self.group)
            return self.C
        return self._chunked(A_panel, B, stream)

    def _chunked(self, A_panel, B, stream):
        self._check(A_panel, B)
        rc, cur = self.rc, self._stream(stream)
        for i in range(self.chunks):
            lo = min(self.rows, i * rc)
            hi = min(self.rows, lo + rc)
            if hi > lo:
                self.compute(A_panel[lo:hi], B, self.mine[i, :hi - lo], hi - lo, self.N, self.K, cur)
            if self.is_cuda:
                ev = torch.cuda.Event()
                ev.record(cur)
                self.comm.wait_event(ev)
                with torch.cuda.stream(self.comm):
                    dist.all_gather_into_tensor(self.stage[i].view(-1, self.N), self.mine[i], group=self.group)
            else:
                dist.all_gather_into_tensor(self.stage[i].view(-1, self.N), self.mine[i], group=self.group)
        if self.is_cuda:
            done = torch.cuda.Event()
            done.record(self.comm)
            cur.wait_event(done)
        # stage[chunk][rank][row] -> C_pad[rank * R + chunk * rc + row]
        full = self.stage.permute(1, 0, 2, 3).reshape(self.world, self.chunks * rc, self.N)[:, :self.R]
        if self.is_cuda:
            with torch.cuda.stream(cur):
                self.C_pad.view(self.world, self.R, self.N).copy_(full)
        else:
            self.C_pad.view(self.world, self.R, self.N).copy_(full)
        return self.C
