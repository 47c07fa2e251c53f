// sb_noalloc.cu -- decode attention that needs no caller-provided scratch.
//
// sb_attn_decode() asks its caller for two small scratch buffers (the
// split-T partial results and one completion ticket per KV head).  Some
// callers cannot allocate device memory at all: hosts that size their whole
// device budget once at start-up (the reference itself targets a 4 GB
// Tegra whose engines allocate everything in gpu_setup and never again),
// plugins inside a framework that owns every allocation and hands a kernel
// only its input and output buffers, and latency-critical decode loops
// that must not enter an allocator between tokens.  For them,
// sb_attn_decode_noalloc() keeps that scratch in a fixed array compiled into
// this library instead.
//
// Limits: T <= SB_NOALLOC_MAX_T (2048) cached positions and at most
// SB_NOALLOC_MAX_HEADS (16) query heads and KV heads; larger requests are
// rejected with SB_ERR_ARG before anything is launched.  The array holds
// 16 heads x 128 splits x 66 floats of partials plus 16 tickets (~528 KiB)
// and stays resident on every GPU that loads the library until the process
// exits.
//
// Set-up: the first call in a CUDA context (a device's primary context, or a
// context the host created itself) looks up the array's device address with
// cudaGetSymbolAddress while that context is current (one lookup per
// context, cached); make that first call before any stream capture begins.
// Every call shares the one array and it keeps the previous call's
// contents: each call clears the tickets it uses (they must start at zero)
// on its stream before launching.  Calls that can overlap on the GPU (two
// streams, or two threads) race on the array and must be serialised by the
// caller.
#include <cuda_runtime.h>
#include <pthread.h>

#include "../csrc/sb_attn.cuh"
#include "sb_internal.h"

#define SB_NOALLOC_MAX_T 2048
#define SB_NOALLOC_MAX_HEADS 16
#define SB_NOALLOC_MAX_SPLITS (SB_NOALLOC_MAX_T / 16)
#define SB_NOALLOC_PART_FLOATS (SB_NOALLOC_MAX_HEADS * SB_NOALLOC_MAX_SPLITS * (SB_ATTN_HD + 2))
#define SB_NOALLOC_TICKETS SB_NOALLOC_MAX_HEADS

// partials first, then the tickets (read as unsigned)
static __device__ __align__(256) float sb_noalloc_scratch[SB_NOALLOC_PART_FLOATS + SB_NOALLOC_TICKETS];

template <int G>
__global__ void attn_decode_noalloc_kernel(const float *__restrict__ q, const float *__restrict__ kc,
                                           const float *__restrict__ vc, int T, float *__restrict__ out,
                                           float *__restrict__ scratch, int kv_stride, float scale,
                                           int max_splits) {
    unsigned *tickets = reinterpret_cast<unsigned *>(scratch + SB_NOALLOC_PART_FLOATS);
    attn_decode_body<G>(q, kc, vc, T, out, scratch, tickets, kv_stride, scale, max_splits);
}

// The array exists once per CUDA context that loads this library's module
// (the primary context of a device, or any context a host created with
// cuCtxCreate, as the reference's hosts do), so its address is looked up --
// and cached -- per context.  Contexts are told apart by cuCtxGetId, which
// is unique for the life of the process, so a context created after another
// was destroyed never inherits the old context's address.
#define SB_NOALLOC_MAX_CONTEXTS 64
static unsigned long long scratch_ctx_id[SB_NOALLOC_MAX_CONTEXTS];
static float *scratch_addr[SB_NOALLOC_MAX_CONTEXTS];
static int scratch_n;
static pthread_mutex_t scratch_lock = PTHREAD_MUTEX_INITIALIZER;

static int device_scratch(float **out) {
    // the library's context rule: the calling thread's current context, else
    // device 0's primary context made current
    const sb_ctx *c = sb_ctx_get();
    if (!c) return SB_ERR_STATE;
    const unsigned long long id = c->ctx_id;
    float *p = nullptr;
    pthread_mutex_lock(&scratch_lock);
    for (int i = 0; i < scratch_n; i++)
        if (scratch_ctx_id[i] == id) p = scratch_addr[i];
    if (!p && scratch_n < SB_NOALLOC_MAX_CONTEXTS) {
        void *a = nullptr;
        if (cudaGetSymbolAddress(&a, sb_noalloc_scratch) == cudaSuccess && a) {
            p = static_cast<float *>(a);
            scratch_ctx_id[scratch_n] = id;
            scratch_addr[scratch_n++] = p;
        }
    }
    pthread_mutex_unlock(&scratch_lock);
    if (!p)
        return sb_fail(SB_ERR_STATE, "cudaGetSymbolAddress(sb_noalloc_scratch) failed (or more than 64 contexts)",
                       __FILE__, __LINE__);
    *out = p;
    return 0;
}

extern "C" int sb_attn_decode_noalloc(const float *q, const float *kc, const float *vc, float *out, int T, int NH,
                                      int NKV, int HD, int kv_stride, float scale, void *stream) {
    if (!q || !kc || !vc || !out) return sb_fail(SB_ERR_ARG, "null pointer", __FILE__, __LINE__);
    if (T < 1 || HD != 64 || NKV <= 0 || NH % NKV != 0 || kv_stride < NKV * HD || kv_stride % 2 != 0)
        return sb_fail(SB_ERR_ARG, "attention: need T >= 1, HD == 64, NH % NKV == 0", __FILE__, __LINE__);
    const int G = NH / NKV;
    if (G != 1 && G != 7) return sb_fail(SB_ERR_ARG, "attention: NH/NKV must be 1 or 7", __FILE__, __LINE__);
    if (T > SB_NOALLOC_MAX_T)
        return sb_fail(SB_ERR_ARG, "sb_attn_decode_noalloc: T exceeds the static scratch limit of 2048 positions",
                       __FILE__, __LINE__);
    if (NH > SB_NOALLOC_MAX_HEADS)
        return sb_fail(SB_ERR_ARG, "sb_attn_decode_noalloc: more than 16 heads exceeds the static scratch",
                       __FILE__, __LINE__);
    float *scratch = nullptr;
    int rc = device_scratch(&scratch);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // tickets must start at zero; earlier calls leave them zeroed, but a call
    // that was aborted may not have
    cudaError_t e = cudaMemsetAsync(scratch + SB_NOALLOC_PART_FLOATS, 0, sizeof(unsigned) * NKV, s);
    if (e != cudaSuccess) return sb_fail(SB_ERR_STATE, cudaGetErrorString(e), __FILE__, __LINE__);
    const int max_splits = (T + 15) / 16;
    const dim3 grid(NKV, max_splits);
    if (G == 7)
        attn_decode_noalloc_kernel<7><<<grid, SB_ATTN_THREADS, 0, s>>>(q, kc, vc, T, out, scratch, kv_stride, scale,
                                                                      max_splits);
    else
        attn_decode_noalloc_kernel<1><<<grid, SB_ATTN_THREADS, 0, s>>>(q, kc, vc, T, out, scratch, kv_stride, scale,
                                                                      max_splits);
    e = cudaGetLastError();
    if (e != cudaSuccess) return sb_fail(SB_ERR_STATE, cudaGetErrorString(e), __FILE__, __LINE__);
    return 0;
}
