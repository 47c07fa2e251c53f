// tc_kernels.cu -- the "tc" module image (sm_100a cubin): 5th-generation
// tensor-core (tcgen05) kernels of this package.
//
// gemm_hh_tc: Y[b][n] = sum_k W[n][k] * X[b][k] for a batch of B <= 256
// fp16 activation rows against fp16 weights, FP32 accumulation -- the
// batched-decode / prefill form of the reference's fp16 GEMV (gemv_h,
// gpu-llm/engine/qwen_kernels.cu:34-70, one activation vector per launch).
// At batch 16 the CUDA-core form needs ~100 TFLOP/s of FP32 FMA to keep up
// with HBM (above the FP32 peak), so the product runs on the tensor pipe:
//   * one CTA per (128-row tile of W, K-range) work item; 6 warps:
//       warp 4 lane 0  TMA producer: W box {64 k, 128 rows} and X box
//                      {64 k, N rows}, 128-byte swizzle, into a 4-stage ring
//                      (full[s] mbarriers with transaction counts),
//       warp 5 lane 0  MMA issuer: tcgen05.mma kind::f16, M=128, N=round16(B),
//                      K=16 per instruction, accumulator in TMEM; each stage
//                      is released with tcgen05.commit -> empty[s],
//       warps 0-3      epilogue: tcgen05.ld of the 128 x N accumulator (warp
//                      w owns TMEM lanes 32w..32w+31 = W rows), stores to Y
//                      (or to the split-K workspace);
//   * rows beyond N and k beyond K are zero-filled by TMA, so any shape with
//     K % 8 == 0 works;
//   * split-K for short weight matrices (few row tiles): partials go to a
//     workspace [splits][B][N] and gemm_splitk_reduce adds them in split
//     order (deterministic).
// Every wait is bounded: on a timeout the kernel raises tc_err, stops
// issuing, waits (bounded) for its copies and MMAs in flight, frees its TMEM
// and returns.
#include <cuda.h>

#include "sb_common.cuh"

namespace tck {
constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr int THREADS = 192;
constexpr long SPIN = 1L << 26;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB per W stage
}  // namespace tck

__device__ int tc_err;  // nonzero after a wait timed out (read and cleared by the host)

namespace tck {
SB_DEV unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
SB_DEV void mbar_init(uint64_t *mb, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mb)), "r"(count) : "memory");
}
SB_DEV void mbar_expect_tx(uint64_t *mb, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mb)), "r"(bytes) : "memory");
}
SB_DEV bool mbar_wait(uint64_t *mb, unsigned ph) {
    for (long spin = 0; spin < SPIN; spin++) {
        unsigned done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(mb)), "r"(ph)
            : "memory");
        if (done) return true;
        if ((spin & 1023) == 1023 && *(volatile int *)&tc_err) return false;
    }
    atomicExch(&tc_err, 1);
    return false;
}
SB_DEV void tma_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *mb) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tm), "r"(x), "r"(y), "r"(smem_u32(mb))
        : "memory");
}
// K-major operand tile of `rows` x 64 fp16 (128-byte rows) written by TMA
// with the 128-byte swizzle: 8-row atoms 1024 bytes apart.
SB_DEV uint64_t sw128_desc(const void *p) {
    const uint64_t addr = smem_u32(p);
    return ((addr >> 4) & 0x3fffull)            // start address
           | (1ull << 16)                       // leading byte offset (unused for swizzled K-major)
           | ((1024ull >> 4) << 32)             // stride byte offset: 8 rows x 128 B
           | (1ull << 46)                       // descriptor version (sm_100)
           | (2ull << 61);                      // 128-byte swizzle
}
// kind::f16 instruction descriptor: f16 A and B, K-major both, f32 D.
SB_DEV uint32_t idesc_f16(int n) {
    return (1u << 4)                            // D format f32
           | ((uint32_t)(n >> 3) << 17)         // N
           | ((uint32_t)(BM >> 4) << 24);       // M = 128
}
SB_DEV void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
            d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
SB_DEV void mma_commit(uint64_t *mb) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(mb))
                 : "memory");
}
SB_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
}  // namespace tck

// grid: items = row_tiles * splits (blockIdx.x = tile * splits + split);
// block tck::THREADS; dynamic smem: 1024 (alignment) + STAGES * (16 KB + n_pad * 128) + 256.
// Output: splits == 1 -> Y[b * N + n]; else ws[(split * B + b) * N + n].
extern "C" __global__ void __launch_bounds__(tck::THREADS, 1)
    gemm_hh_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
               float *__restrict__ Y, float *__restrict__ ws, int N, int K, int B, int n_pad, int splits) {
    using namespace tck;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int b_bytes = n_pad * BK * 2;
    unsigned char *a_st = smem;                                  // STAGES x 16 KB
    unsigned char *b_st = smem + STAGES * A_BYTES;               // STAGES x n_pad x 128 B (1024-aligned: n_pad % 16 == 0... see host)
    uint64_t *bars = reinterpret_cast<uint64_t *>(b_st + STAGES * b_bytes);
    uint64_t *full = bars, *empty = bars + STAGES, *accb = bars + 2 * STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x / splits, split = blockIdx.x % splits;
    const int m0 = tile * BM;
    const int nchunks = (K + BK - 1) / BK;
    const int c0 = (int)((long)nchunks * split / splits), c1 = (int)((long)nchunks * (split + 1) / splits);
    const uint32_t tmem_cols = n_pad <= 32 ? 32 : (n_pad <= 64 ? 64 : (n_pad <= 128 ? 128 : 256));

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accb, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // TMEM accumulator: 128 lanes x tmem_cols fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 4 && lane == 0) {
        // ---- TMA producer
        const unsigned tx = (unsigned)(A_BYTES + b_bytes);
        int issued = 0;
        bool ok = true;
        for (int c = c0; c < c1 && ok; c++, issued++) {
            const int s = issued % STAGES;
            if (issued >= STAGES) ok = mbar_wait(&empty[s], ((issued / STAGES) - 1) & 1);
            if (!ok) break;
            mbar_expect_tx(&full[s], tx);
            tma_2d(a_st + (size_t)s * A_BYTES, &tm_w, c * BK, m0, &full[s]);
            tma_2d(b_st + (size_t)s * b_bytes, &tm_x, c * BK, 0, &full[s]);
        }
        // every stage issued must have landed before this CTA may exit
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; i++) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    } else if (warp == 5 && lane == 0) {
        // ---- MMA issuer
        const uint32_t idesc = idesc_f16(n_pad);
        int used = 0;
        for (int c = c0; c < c1; c++, used++) {
            const int s = used % STAGES;
            if (!mbar_wait(&full[s], (used / STAGES) & 1)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t da = sw128_desc(a_st + (size_t)s * A_BYTES), db = sw128_desc(b_st + (size_t)s * b_bytes);
#pragma unroll
            for (int k = 0; k < BK / 16; k++)  // +32 bytes per K=16 step inside the swizzled 128-byte rows
                mma_f16(tmem, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (c > c0 || k > 0) ? 1u : 0u);
            mma_commit(&empty[s]);
        }
        mma_commit(accb);  // arrives once every MMA issued above has completed
    } else if (warp < 4) {
        // ---- epilogue: wait for the accumulator, TMEM -> registers -> global
        const bool ok = mbar_wait(accb, 0);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int n = m0 + warp * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        for (int col = 0; col < n_pad; col += 16) {
            float v[16];
            tmem_ld16(lane_base + (uint32_t)col, v);
            if (!ok || c1 <= c0) continue;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int b = col + j;
                if (b < B && n < N) {
                    if (splits == 1) Y[(size_t)b * N + n] = v[j];
                    else ws[((size_t)split * B + b) * N + n] = v[j];
                }
            }
        }
        if (c1 <= c0 && ok) {  // an empty K-range contributes zeros
            for (int b = 0; b < B; b++)
                if (n < N) {
                    if (splits == 1) Y[(size_t)b * N + n] = 0.f;
                    else ws[((size_t)split * B + b) * N + n] = 0.f;
                }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
    }
}

// Y[b][n] = sum over splits s (in order) of ws[s][b][n].
extern "C" __global__ void gemm_splitk_reduce(const float *__restrict__ ws, float *__restrict__ Y, long total,
                                              int splits) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int s = 0; s < splits; s++) acc += ws[(size_t)s * total + i];
        Y[i] = acc;
    }
}
