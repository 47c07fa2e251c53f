"""ctypes access to the CPU oracle (oracle/liboracle.so) and to the reference's
own C compiled under oracle/_ref/ -- test infrastructure only."""
import ctypes
import os
import subprocess

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(REPO, "oracle")
ORACLE_LIB = os.path.join(ORACLE_DIR, "liboracle.so")
REF_DIR = os.path.join(ORACLE_DIR, "_ref")

_orc = None


def _f32p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def oracle():
    global _orc
    if _orc is not None:
        return _orc
    if not os.path.exists(ORACLE_LIB):
        subprocess.run(["make", "-C", ORACLE_DIR, "liboracle.so"], check=True, capture_output=True)
    L = ctypes.CDLL(ORACLE_LIB)
    P, I, F, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
    L.orc_h2f.restype = F
    L.orc_h2f.argtypes = [ctypes.c_uint16]
    L.orc_sgemm_rows.argtypes = [P, P, P, I, I, I, I, I, I]
    L.orc_sgemm_rows.restype = None
    L.orc_sgemm_bad_cells.argtypes = [P, P, ctypes.c_size_t]
    L.orc_sgemm_bad_cells.restype = I
    L.orc_freivalds.argtypes = [P, P, P, I, I, I, ctypes.c_uint64, I]
    L.orc_freivalds.restype = D
    L.orc_gemv_f32.argtypes = [P, P, P, P, I, I, I]
    L.orc_gemv_multi_f32.argtypes = [P, P, P, P, I, I, I, I]
    L.orc_gemv_h.argtypes = [P, P, P, P, I, I, I]
    L.orc_rmsnorm.argtypes = [P, P, P, I, F]
    L.orc_layernorm.argtypes = [P, P, P, P, I, F]
    L.orc_rope.argtypes = [P, P, P, I, I, I, I]
    L.orc_swiglu.argtypes = [P, P, P, I]
    L.orc_gelu.argtypes = [P, P, I]
    L.orc_attn_qwen.argtypes = [P, P, P, P, I, I, I, I, I, F]
    L.orc_attn_gpt2.argtypes = [P, P, P, P, I, I, I, I, F]
    for n in ("qwen", "gpt2"):
        getattr(L, f"orc_{n}_open").restype = P
        getattr(L, f"orc_{n}_open").argtypes = [ctypes.c_char_p, I]
        getattr(L, f"orc_{n}_reset").argtypes = [P]
        getattr(L, f"orc_{n}_forward").argtypes = [P, I, I, I, P, I]
        getattr(L, f"orc_{n}_residual").argtypes = [P]
        getattr(L, f"orc_{n}_residual").restype = P
        getattr(L, f"orc_{n}_close").argtypes = [P]
        getattr(L, f"orc_{n}_kv").argtypes = [P, I]
        getattr(L, f"orc_{n}_kv").restype = P
    L.orc_argmax.argtypes = [P, I]
    L.orc_argmax.restype = I
    _orc = L
    return L


NTHREADS = max(1, min(64, os.cpu_count() or 1))


def sgemm(A, B, row0=0, row1=None, nthreads=NTHREADS):
    M, K = A.shape
    N = B.shape[1]
    row1 = M if row1 is None else row1
    C = np.zeros((M, N), dtype=np.float32)
    oracle().orc_sgemm_rows(_f32p(A), _f32p(B), _f32p(C), M, N, K, row0, row1, nthreads)
    return C


def sgemm_bad_cells(C, ref):
    """Cells outside the harness tolerance (gpu_workload.c:99-101)."""
    C, ref = np.ascontiguousarray(C, dtype=np.float32), np.ascontiguousarray(ref, dtype=np.float32)
    return oracle().orc_sgemm_bad_cells(_f32p(C), _f32p(ref), C.size)


def freivalds(A, B, C, seed=7):
    M, K = A.shape
    N = B.shape[1]
    return oracle().orc_freivalds(_f32p(A), _f32p(B), _f32p(C), M, N, K, seed, NTHREADS)


def gemv_f32(W, x, bias=None):
    N, K = W.shape
    y = np.zeros(N, dtype=np.float32)
    oracle().orc_gemv_f32(_f32p(W), _f32p(x), _f32p(bias), _f32p(y), K, N, NTHREADS)
    return y


def gemv_multi_f32(W, X, bias=None):
    N, K = W.shape
    T = X.shape[0]
    Y = np.zeros((T, N), dtype=np.float32)
    oracle().orc_gemv_multi_f32(_f32p(W), _f32p(X), _f32p(bias), _f32p(Y), K, N, T, NTHREADS)
    return Y


def gemv_h(W16, x, bias=None):
    N, K = W16.shape
    y = np.zeros(N, dtype=np.float32)
    oracle().orc_gemv_h(_f32p(W16), _f32p(x), _f32p(bias), _f32p(y), K, N, NTHREADS)
    return y


def h2f(bits):
    """Vectorised reference fp16 decode of uint16 bits (qwen_engine.c:90-98):
    exponent 0 -> 0, and no inf/NaN case (exponent 31 decodes to a finite
    value, as in the reference)."""
    h = np.asarray(bits, dtype=np.uint16).astype(np.uint32)
    e = (h >> 10) & 0x1F
    u = ((h & 0x8000) << 16) | ((e + 112) << 23) | ((h & 0x3FF) << 13)
    u[e == 0] = 0
    return u.astype(np.uint32).view(np.float32)


def rmsnorm(x, w16, eps):
    y = np.zeros_like(x)
    oracle().orc_rmsnorm(_f32p(x), _f32p(w16), _f32p(y), x.size, eps)
    return y


def layernorm(x, w, b, eps):
    y = np.zeros_like(x)
    oracle().orc_layernorm(_f32p(x), _f32p(w), _f32p(b), _f32p(y), x.size, eps)
    return y


def rope(x, cosT, sinT, T, H, HD, pos0):
    y = x.copy()
    oracle().orc_rope(_f32p(y), _f32p(cosT), _f32p(sinT), T, H, HD, pos0)
    return y


def swiglu(g, u):
    y = np.zeros_like(g)
    oracle().orc_swiglu(_f32p(g), _f32p(u), _f32p(y), g.size)
    return y


def gelu(x):
    y = np.zeros_like(x)
    oracle().orc_gelu(_f32p(x), _f32p(y), x.size)
    return y


def attn_qwen(q, kc, vc, T, NH, NKV, HD, kv_stride, scale):
    out = np.zeros(NH * HD, dtype=np.float32)
    oracle().orc_attn_qwen(_f32p(q), _f32p(kc), _f32p(vc), _f32p(out), T, NH, NKV, HD, kv_stride, scale)
    return out


def attn_gpt2(q, kc, vc, T, NH, HD, kv_stride, scale):
    out = np.zeros(NH * HD, dtype=np.float32)
    oracle().orc_attn_gpt2(_f32p(q), _f32p(kc), _f32p(vc), _f32p(out), T, NH, HD, kv_stride, scale)
    return out


class Model:
    """Oracle decode model over a weight file (name: 'qwen' or 'gpt2')."""

    def __init__(self, name, path, ctx, vocab):
        self.name = name
        self.vocab = vocab
        L = oracle()
        self.h = getattr(L, f"orc_{name}_open")(str(path).encode(), ctx)
        if not self.h:
            raise RuntimeError(f"oracle could not open {path}")

    def forward(self, token, pos, want_logits=True, nthreads=NTHREADS):
        logits = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        getattr(oracle(), f"orc_{self.name}_forward")(self.h, token, pos, 1 if want_logits else 0,
                                                      _f32p(logits), nthreads)
        return logits

    def reset(self):
        getattr(oracle(), f"orc_{self.name}_reset")(self.h)

    def kv(self, ctx, layers, width):
        """The KV cache as one writable (2, layers, ctx, width) FP32 view:
        [0] keys, [1] values (the oracle keeps them as two arrays, so this
        returns a pair of (layers, ctx, width) views)."""
        out = []
        for which in (0, 1):
            ptr = getattr(oracle(), f"orc_{self.name}_kv")(self.h, which)
            buf = (ctypes.c_float * (layers * ctx * width)).from_address(ptr)
            out.append(np.ctypeslib.as_array(buf).reshape(layers, ctx, width))
        return out

    def close(self):
        if self.h:
            getattr(oracle(), f"orc_{self.name}_close")(self.h)
            self.h = None


def greedy(model, prompt, n_gen, eos=()):
    """The reference prime-then-generate loop (qwen_engine.c:523-548) on the
    oracle: returns prompt + generated ids and the per-step logits."""
    ids = list(prompt)
    logits = None
    for p, t in enumerate(prompt):
        logits = model.forward(t, p, p == len(prompt) - 1)
    nxt = int(np.argmax(logits))
    ids.append(nxt)
    steps = [logits]
    for _ in range(n_gen):
        if nxt in eos:
            break
        logits = model.forward(nxt, len(ids) - 1, True)
        steps.append(logits)
        nxt = int(np.argmax(logits))
        ids.append(nxt)
    return ids, steps


# ---------------------------------------------------------------- reference (oracle/_ref)
def ref_available():
    return all(os.path.exists(os.path.join(REF_DIR, f)) for f in
               ("libref_qwen.so", "libref_gpt2.so", "gpu_workload_emu", "gemv_test_emu"))


def ref_lib(name):
    L = ctypes.CDLL(os.path.join(REF_DIR, f"libref_{name}.so"))
    P, I = ctypes.c_void_p, ctypes.c_int
    getattr(L, f"ref_{name}_load").argtypes = [ctypes.c_char_p]
    getattr(L, f"ref_{name}_forward").argtypes = [I, I, I, P]
    getattr(L, f"ref_{name}_residual").argtypes = [P]
    if name == "qwen":
        L.ref_gemv_h.argtypes = [P, P, P, P, I, I]
        L.ref_rms.argtypes = [P, P, P, I]
        L.ref_h2f.argtypes = [ctypes.c_uint16]
        L.ref_h2f.restype = ctypes.c_float
        L.ref_sample_token.argtypes = [P, P, I]
        L.ref_sample_token.restype = I
        L.ref_sampler_seed.argtypes = [ctypes.c_uint]
    else:
        L.ref_gemv.argtypes = [P, P, P, P, I, I]
        L.ref_ln.argtypes = [P, P, P, P]
    return L
