"""ctypes binding of libswitch_b200 (the C-ABI declared in include/switch_b200.h).

This is how Python callers (the tests, bench.py) reach the sm_100a kernels:
every call goes through the shared library's extern "C" entry points with
plain device pointers, sizes and a CUstream handle.  PyTorch is only used by
callers for device memory and streams; pass ``tensor.data_ptr()`` and
``torch.cuda.current_stream().cuda_stream``.

There is no fallback: if the library or a CUDA driver is missing, loading
fails loudly.
"""
import ctypes
import ctypes.util
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(_HERE, "lib")
BIN_DIR = os.path.join(_HERE, "bin")
LIB_PATH = os.path.join(LIB_DIR, "libswitch_b200.so")
CUBINS = {m: os.path.join(LIB_DIR, m + ".cubin") for m in ("switch_gpu", "gemv", "gpt2", "qwen", "tc")}

MODEL_QWEN = 1
MODEL_GPT2 = 2
FLAG_NO_GRAPH = 1
FLAG_NO_PDL = 2
FLAG_MULTI_KERNEL = 4
FLAG_NO_PREFILL = 8
FLAG_MK_V1 = 16  # Qwen: the earlier persistent step kernel (A/B and regression tests)
GEN_STOP_EOS = 1

QWEN = dict(V=151936, C=896, NL=24, NH=14, NKV=2, HD=64, FC=4864, CTX_FILE=8192,
            FILE_BYTES=990162688, EOT=151643, IM_END=151645)
GPT2 = dict(V=50257, C=768, NL=12, NH=12, HD=64, FC=3072, CTX=1024, TOTAL_FLOATS=124439808, EOT=50256)

_lib = None
_cuda_is_stub = False


def _load_driver():
    """Make libcuda.so.1 resolvable for libswitch_b200's NEEDED entry.

    On a GPU machine this is the real driver.  On a machine without one the
    toolkit's link stub is loaded instead so the library can be inspected
    (symbols, module images); every CUDA call then fails with an error."""
    global _cuda_is_stub
    try:
        return ctypes.CDLL("libcuda.so.1", mode=ctypes.RTLD_GLOBAL)
    except OSError:
        stub = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64", "stubs", "libcuda.so")
        _cuda_is_stub = True
        return ctypes.CDLL(stub, mode=ctypes.RTLD_GLOBAL)


def driver_is_stub():
    lib()
    return _cuda_is_stub


def _sig(f, res, *args):
    f.restype = res
    f.argtypes = list(args)


def lib():
    """Load and prototype libswitch_b200.so (once)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it first (make -C switch-l4t-gpu_b200)")
    _load_driver()
    L = ctypes.CDLL(LIB_PATH)
    P, I, F, D, U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_uint64
    _sig(L.sb_init, I, I)
    _sig(L.sb_last_error, ctypes.c_char_p)
    _sig(L.sb_module_image, I, ctypes.c_char_p, ctypes.POINTER(P), ctypes.POINTER(ctypes.c_size_t))
    _sig(L.sb_sm_count, I)
    _sig(L.sb_sgemm, I, P, P, P, I, I, I, P)
    _sig(L.sb_sgemm_rows, I, P, P, P, I, I, I, I, I, P)
    _sig(L.sb_sgemm_multi, I, P, P, ctypes.POINTER(P), I, I, I, I, P)
    _sig(L.sb_ipc_export, I, P, P, ctypes.POINTER(ctypes.c_size_t))
    _sig(L.sb_ipc_open, I, P, ctypes.c_size_t, ctypes.POINTER(P))
    _sig(L.sb_ipc_close, I, P, ctypes.c_size_t)
    _sig(L.sb_membw_read4, I, P, P, I, I, I, P)
    _sig(L.sb_fma_peak, I, P, I, I, P, ctypes.POINTER(D))
    _sig(L.sb_gemv_f32, I, P, P, P, P, I, I, P)
    _sig(L.sb_gemv_multi_f32, I, P, P, P, P, I, I, I, P)
    _sig(L.sb_gemv_h, I, P, P, P, P, I, I, P)
    _sig(L.sb_gemv_hh, I, P, P, P, I, I, I, P)
    _sig(L.sb_gemm_hh, I, P, P, P, I, I, I, P)
    _sig(L.sb_tc_error, I, P)
    _sig(L.sb_sgemm_3xtf32, I, P, P, P, I, I, I, P)
    _sig(L.sb_sgemm_3xtf32_multi, I, P, P, ctypes.POINTER(P), I, I, I, I, P)
    _sig(L.sb_rmsnorm, I, P, P, P, I, F, I, P)
    _sig(L.sb_rope, I, P, P, P, I, I, I, I, P)
    _sig(L.sb_swiglu, I, P, P, P, I, P)
    _sig(L.sb_attn_decode, I, P, P, P, P, I, I, I, I, I, F, P, P, P)
    _sig(L.sb_attn_decode_noalloc, I, P, P, P, P, I, I, I, I, I, F, P)
    _sig(L.sb_layernorm, I, P, P, P, P, I, F, I, P)
    _sig(L.sb_gelu, I, P, P, I, P)
    _sig(L.sb_tc_set_test_skip, I, I)
    _sig(L.sb_sgemm_tma, I, P, P, P, I, I, I, P)
    _sig(L.sb_nccl_unique_id, I, P)
    _sig(L.sb_nccl_comm_init, I, P, I, P, I, ctypes.c_double)
    _sig(L.sb_nccl_comm_destroy, I, P, ctypes.c_double)
    _sig(L.sb_nccl_abort, I, P)
    _sig(L.sb_sgemm_panel_allgather, I, P, P, P, I, I, I, I, I, P, I, P)
    _sig(L.sb_nccl_wait, I, P, P, ctypes.c_double)
    _sig(L.sb_engine_create, P, I, ctypes.c_char_p, I, ctypes.c_uint)
    _sig(L.sb_engine_destroy, None, P)
    _sig(L.sb_engine_reset, I, P)
    _sig(L.sb_engine_kv_cache, I, P, P, P, P, P, P)
    _sig(L.sb_engine_step_kernel, ctypes.c_char_p, P)
    _sig(L.sb_engine_forward, I, P, I, I, I, P)
    _sig(L.sb_engine_generate, I, P, P, I, I, P, ctypes.POINTER(I), ctypes.c_uint)
    _sig(L.sb_engine_begin, I, P, P, I, I, ctypes.c_uint)
    _sig(L.sb_engine_steps, I, P, I, I)
    _sig(L.sb_engine_prefill, I, P, I)
    _sig(L.sb_engine_finish, I, P, P, ctypes.POINTER(I))
    _sig(L.sb_engine_stream, P, P)
    _sig(L.sb_engine_logits, I, P, ctypes.POINTER(P), ctypes.POINTER(I))
    _sig(L.sb_engine_launches_per_step, I, P, I)
    _sig(L.sb_engine_step_bytes, D, P)
    _sig(L.sb_engine_uses_persistent_kernel, I, P)
    _sig(L.sb_engine_set_trace, I, P, P)
    _sig(L.sb_engine_set_test_stall, I, P, I)
    _sig(L.sb_engine_profile, I, P, I, I, P, ctypes.c_size_t, ctypes.POINTER(F), ctypes.POINTER(D))
    _sig(L.sb_sample_token, I, P, I, P, I, F, I, F, F, ctypes.POINTER(ctypes.c_uint32), P)
    _sig(L.sb_topk_penalized, I, P, I, P, I, F, F, I, P, P, P)
    _sig(L.sb_sample_topk, I, P, P, I, F, ctypes.POINTER(ctypes.c_uint32))
    _sig(L.sb_engine_sample, I, P, I, F, I, F, F, ctypes.POINTER(ctypes.c_uint32))
    _sig(L.sb_synth_weights, ctypes.c_long, I, ctypes.c_char_p, U64)
    _sig(L.sb_synth_ids, None, P, I, I, U64)
    _sig(L.sb_synth_uniform, None, P, ctypes.c_size_t, F, F, U64)
    _sig(L.sb_synth_normal_h, None, P, ctypes.c_size_t, F, U64)
    _lib = L
    return L


class SbError(RuntimeError):
    pass


def check(rc):
    if rc != 0:
        raise SbError(f"libswitch_b200 error {rc}: {lib().sb_last_error().decode()}")
    return rc


def _p(x):
    """Device pointer of a torch tensor / int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _s(stream):
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ---------------------------------------------------------------- ops
def init(device=0):
    check(lib().sb_init(device))


def sm_count():
    return lib().sb_sm_count()


def module_image(name):
    p = ctypes.c_void_p()
    n = ctypes.c_size_t()
    check(lib().sb_module_image(name.encode(), ctypes.byref(p), ctypes.byref(n)))
    return ctypes.string_at(p, n.value)


def sgemm(A, B, C, M, N, K, stream=None):
    check(lib().sb_sgemm(_p(A), _p(B), _p(C), M, N, K, _s(stream)))


def sgemm_tma(A, B, C, M, N, K, stream=None):
    """The TMA-staged CUDA-core SGEMM (bit-identical to sgemm)."""
    check(lib().sb_sgemm_tma(_p(A), _p(B), _p(C), M, N, K, _s(stream)))


def sgemm_rows(A, B, C, M, N, K, row0, row1, stream=None):
    check(lib().sb_sgemm_rows(_p(A), _p(B), _p(C), M, N, K, row0, row1, _s(stream)))


def sgemm_multi(A, B, outs, M, N, K, stream=None):
    """C = A.B stored into every matrix of `outs` (tensors or raw device
    addresses, local or peer-mapped; at most 8): sb_sgemm_multi."""
    arr = (ctypes.c_void_p * len(outs))(*[_p(c) for c in outs])
    check(lib().sb_sgemm_multi(_p(A), _p(B), arr, len(outs), M, N, K, _s(stream)))


def ipc_export(t):
    """(64-byte CUDA IPC handle of the allocation holding `t`, t's offset in it)."""
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_size_t()
    check(lib().sb_ipc_export(_p(t), h, ctypes.byref(off)))
    return h.raw, off.value


def ipc_open(handle, offset):
    """Device address, in this process, of a buffer another process exported."""
    p = ctypes.c_void_p()
    check(lib().sb_ipc_open(ctypes.create_string_buffer(handle, 64), offset, ctypes.byref(p)))
    return p.value


def ipc_close(addr, offset):
    check(lib().sb_ipc_close(addr, offset))


def membw_read4(buf, out, n4, iters, grid=0, stream=None):
    check(lib().sb_membw_read4(_p(buf), _p(out), n4, iters, grid, _s(stream)))


def fma_peak(out, iters, grid=0, stream=None):
    fl = ctypes.c_double()
    check(lib().sb_fma_peak(_p(out), iters, grid, _s(stream), ctypes.byref(fl)))
    return fl.value


def gemv_f32(W, x, bias, y, K, N, stream=None):
    check(lib().sb_gemv_f32(_p(W), _p(x), _p(bias), _p(y), K, N, _s(stream)))


def gemv_multi_f32(W, X, bias, Y, K, N, T, stream=None):
    check(lib().sb_gemv_multi_f32(_p(W), _p(X), _p(bias), _p(Y), K, N, T, _s(stream)))


def gemv_h(W, x, bias, y, K, N, stream=None):
    check(lib().sb_gemv_h(_p(W), _p(x), _p(bias), _p(y), K, N, _s(stream)))


def gemv_hh(W, X, Y, K, N, B, stream=None):
    check(lib().sb_gemv_hh(_p(W), _p(X), _p(Y), K, N, B, _s(stream)))


def gemm_hh(W, X, Y, K, N, B, stream=None):
    """Tensor-core (tcgen05) Y[b][n] = sum_k W[n][k] X[b][k], B <= 256."""
    check(lib().sb_gemm_hh(_p(W), _p(X), _p(Y), K, N, B, _s(stream)))


def topk_penalized(logits, V, ctx, ctx_len, temperature, rep_penalty, k, idx_out, val_out, stream=None):
    """Device steps 1-3 of the Qwen sampler: the k (id, value) candidates of
    the penalised, temperature-scaled logits (all device tensors)."""
    check(lib().sb_topk_penalized(_p(logits), V, _p(ctx), ctx_len, temperature, rep_penalty, k, _p(idx_out),
                                  _p(val_out), _s(stream)))


def sample_topk(idx, val, top_p, state):
    """Host steps 4-6 on k candidates (numpy int32 / float32 arrays); state:
    ctypes.c_uint32 xorshift state, advanced in place."""
    import numpy as np
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    val = np.ascontiguousarray(val, dtype=np.float32)
    return lib().sb_sample_topk(idx.ctypes.data, val.ctypes.data, len(idx), top_p, ctypes.byref(state))


def sgemm_3xtf32_multi(A, B, outs, M, N, K, stream=None):
    """The 3xTF32 SGEMM stored into every matrix of `outs`: sb_sgemm_3xtf32_multi."""
    arr = (ctypes.c_void_p * len(outs))(*[_p(c) for c in outs])
    check(lib().sb_sgemm_3xtf32_multi(_p(A), _p(B), arr, len(outs), M, N, K, _s(stream)))


def sgemm_3xtf32(A, B, C, M, N, K, stream=None):
    """Opt-in FP32 SGEMM on the TF32 tensor pipe (3xTF32 split)."""
    check(lib().sb_sgemm_3xtf32(_p(A), _p(B), _p(C), M, N, K, _s(stream)))


def tc_error():
    """Read and clear the tensor-core kernels' device error flag."""
    e = ctypes.c_int()
    check(lib().sb_tc_error(ctypes.byref(e)))
    return e.value


def rmsnorm(x, w, y, n, eps, rows=1, stream=None):
    check(lib().sb_rmsnorm(_p(x), _p(w), _p(y), n, eps, rows, _s(stream)))


def rope(x, cosT, sinT, T, H, HD, pos0, stream=None):
    check(lib().sb_rope(_p(x), _p(cosT), _p(sinT), T, H, HD, pos0, _s(stream)))


def swiglu(g, u, y, n, stream=None):
    check(lib().sb_swiglu(_p(g), _p(u), _p(y), n, _s(stream)))


def attn_decode(q, kc, vc, out, T, NH, NKV, HD, kv_stride, scale, part, counters, stream=None):
    check(lib().sb_attn_decode(_p(q), _p(kc), _p(vc), _p(out), T, NH, NKV, HD, kv_stride, scale,
                               _p(part), _p(counters), _s(stream)))


def attn_decode_noalloc(q, kc, vc, out, T, NH, NKV, HD, kv_stride, scale, stream=None):
    """sb_attn_decode without caller scratch (static device array, T <= 2048)."""
    check(lib().sb_attn_decode_noalloc(_p(q), _p(kc), _p(vc), _p(out), T, NH, NKV, HD, kv_stride, scale, _s(stream)))


def layernorm(x, w, b, y, n, eps, rows=1, stream=None):
    check(lib().sb_layernorm(_p(x), _p(w), _p(b), _p(y), n, eps, rows, _s(stream)))


def gelu(x, y, n, stream=None):
    check(lib().sb_gelu(_p(x), _p(y), n, _s(stream)))


# ---------------------------------------------------------------- synthetic inputs
def synth_weights(model, path, seed):
    n = lib().sb_synth_weights(model, str(path).encode(), seed)
    if n < 0:
        raise SbError(f"could not write synthetic weights to {path}")
    return n


def synth_ids(n, vocab, seed):
    arr = (ctypes.c_int * n)()
    lib().sb_synth_ids(arr, n, vocab, seed)
    return list(arr)


def synth_uniform(n, lo, hi, seed):
    import numpy as np
    out = np.empty(n, dtype=np.float32)
    lib().sb_synth_uniform(out.ctypes.data, n, lo, hi, seed)
    return out


def synth_normal_h(n, std, seed):
    import numpy as np
    out = np.empty(n, dtype=np.uint16)
    lib().sb_synth_normal_h(out.ctypes.data, n, std, seed)
    return out


# ---------------------------------------------------------------- engines
class Engine:
    """A decode engine (one model on the current device)."""

    def __init__(self, model, weights_path, max_ctx, flags=0):
        L = lib()
        self.model = model
        self.h = L.sb_engine_create(model, str(weights_path).encode(), max_ctx, flags)
        if not self.h:
            raise SbError(f"engine create failed: {L.sb_last_error().decode()}")
        p = ctypes.c_void_p()
        v = ctypes.c_int()
        check(L.sb_engine_logits(self.h, ctypes.byref(p), ctypes.byref(v)))
        self.logits_ptr = p.value
        self.vocab = v.value

    def close(self):
        if self.h:
            lib().sb_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        check(lib().sb_engine_reset(self.h))

    def forward(self, token, pos, want_logits=True, logits_out=None):
        """Reference gpu_forward contract; logits_out: numpy float32[V] or None."""
        ptr = None if logits_out is None else logits_out.ctypes.data
        check(lib().sb_engine_forward(self.h, token, pos, 1 if want_logits else 0, ptr))

    def sample(self, ctx_len, state, temperature=0.7, top_k=20, top_p=0.8, rep_penalty=1.1):
        """Next token from the last step's device logits with the reference
        sampler's settings (device top-k, host draw); state: ctypes.c_uint32."""
        t = lib().sb_engine_sample(self.h, ctx_len, temperature, top_k, top_p, rep_penalty, ctypes.byref(state))
        if t < 0:
            check(-t)
        return t

    def generate(self, prompt, n_gen, stop_eos=False):
        n_prompt = len(prompt)
        arr = (ctypes.c_int * n_prompt)(*prompt)
        out = (ctypes.c_int * (n_prompt + n_gen + 1))()
        n = ctypes.c_int()
        check(lib().sb_engine_generate(self.h, arr, n_prompt, n_gen, out, ctypes.byref(n),
                                       GEN_STOP_EOS if stop_eos else 0))
        return list(out[: n.value])

    def begin(self, prompt, n_gen, stop_eos=False):
        arr = (ctypes.c_int * len(prompt))(*prompt)
        check(lib().sb_engine_begin(self.h, arr, len(prompt), n_gen, GEN_STOP_EOS if stop_eos else 0))

    def prefill(self, n):
        """Qwen: batched prefill of the first n prompt tokens (after begin)."""
        check(lib().sb_engine_prefill(self.h, n))

    def steps(self, n, with_logits):
        check(lib().sb_engine_steps(self.h, n, 1 if with_logits else 0))

    def finish(self, capacity):
        out = (ctypes.c_int * capacity)()
        n = ctypes.c_int()
        check(lib().sb_engine_finish(self.h, out, ctypes.byref(n)))
        return list(out[: n.value])

    @property
    def stream(self):
        return lib().sb_engine_stream(self.h)

    def set_trace(self, buf):
        check(lib().sb_engine_set_trace(self.h, _p(buf)))

    def set_test_stall(self, cta):
        """Failure-detection test hook: CTA `cta` withholds its layer-0
        outputs (-1: off); see sb_engine_set_test_stall."""
        check(lib().sb_engine_set_test_stall(self.h, cta))

    @property
    def step_kernel(self):
        """Name of the kernel that runs the decode step."""
        return lib().sb_engine_step_kernel(self.h).decode()

    @property
    def persistent(self):
        return bool(lib().sb_engine_uses_persistent_kernel(self.h))

    def kv_cache(self):
        """(device pointer, bytes, layers, max_ctx, width) of the FP32
        [2][layers][max_ctx][width] KV cache."""
        p, nb = ctypes.c_void_p(), ctypes.c_size_t()
        nl, ctx, w = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().sb_engine_kv_cache(self.h, ctypes.byref(p), ctypes.byref(nb), ctypes.byref(nl), ctypes.byref(ctx),
                                       ctypes.byref(w)))
        return p.value, nb.value, nl.value, ctx.value, w.value

    def launches_per_step(self, with_logits=True):
        return lib().sb_engine_launches_per_step(self.h, 1 if with_logits else 0)

    def step_bytes(self):
        return lib().sb_engine_step_bytes(self.h)

    # kernel ids of sb_engine_profile
    K_QKV, K_ATTN, K_O, K_MLP_UP, K_MLP_DOWN, K_LMHEAD = 1, 2, 3, 4, 5, 6

    def profile(self, which, reps, flush=None, flush_bytes=0):
        """(avg ms, algorithmic bytes) of `reps` standalone launches."""
        ms = ctypes.c_float()
        by = ctypes.c_double()
        check(lib().sb_engine_profile(self.h, which, reps, _p(flush), flush_bytes, ctypes.byref(ms), ctypes.byref(by)))
        return ms.value, by.value


if __name__ == "__main__":
    # python sb200.py synth {qwen|gpt2} PATH SEED -- write a seeded synthetic
    # weight file in the reference layout (used by profiling commands).
    import sys
    if len(sys.argv) == 5 and sys.argv[1] == "synth" and sys.argv[2] in ("qwen", "gpt2"):
        model = MODEL_QWEN if sys.argv[2] == "qwen" else MODEL_GPT2
        print(synth_weights(model, sys.argv[3], int(sys.argv[4])), "bytes written to", sys.argv[3])
    else:
        sys.exit("usage: sb200.py synth {qwen|gpt2} PATH SEED")
