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
// Failure-detection test hook (set by the host, sb_tc_set_test_skip): k + 1
// makes every gemm_hh_tc producer stop before issuing its K-chunk k, so the
// MMA issuer's wait for that stage runs out and the kernel reports tc_err;
// 0 = off.
__device__ int tc_test_skip;

namespace tck {
SB_DEV unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
SB_DEV void mbar_init(uint64_t *mb, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mb)), "r"(count) : "memory");
}
SB_DEV void mbar_expect_tx(uint64_t *mb, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mb)), "r"(bytes) : "memory");
}
SB_DEV unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for phase `ph` of an mbarrier.  Gives up after WAIT_NS of
// wall time (or SPIN polls), raising tc_err.  `abortable` waits -- for
// something another role may never deliver once it has stopped -- also
// return early when another thread already raised tc_err; the others (a
// TMA copy or MMA batch this CTA issued, which always completes) keep
// waiting, so a CTA never frees shared or tensor memory under work in flight.
constexpr unsigned long long WAIT_NS = 2000000000ull;
SB_DEV bool mbar_wait(uint64_t *mb, unsigned ph, bool abortable = true) {
    unsigned long long t0 = 0;
    for (long spin = 0; spin < SPIN; spin++) {
        unsigned done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(mb)), "r"(ph)
            : "memory");
        if (done) return true;
        if ((spin & 1023) == 1023) {
            if (abortable && *(volatile int *)&tc_err) return false;
            const unsigned long long t = gtimer();
            if (t0 == 0) t0 = t;
            else if (t - t0 > WAIT_NS) break;
        }
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
        const int skip = tc_test_skip - 1;  // test hook: -1 = off
        int issued = 0;
        bool ok = true;
        for (int c = c0; c < c1 && ok; c++, issued++) {
            if (issued == skip) break;  // withhold this stage: the MMA issuer's wait runs out
            const int s = issued % STAGES;
            if (issued >= STAGES) ok = mbar_wait(&empty[s], ((issued / STAGES) - 1) & 1);
            if (!ok) break;
            mbar_expect_tx(&full[s], tx);
            tma_2d(a_st + (size_t)s * A_BYTES, &tm_w, c * BK, m0, &full[s]);
            tma_2d(b_st + (size_t)s * b_bytes, &tm_x, c * BK, 0, &full[s]);
        }
        // every stage issued must have landed before this CTA may exit
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; i++)
            mbar_wait(&full[i % STAGES], (i / STAGES) & 1, false);
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
        // ---- epilogue: wait for the accumulator (the MMA issuer always
        // commits it, also after giving up, once its MMAs have drained),
        // TMEM -> registers -> global; nothing is stored after a timeout
        const bool ok = mbar_wait(accb, 0, false) && !*(volatile int *)&tc_err;
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

// The same with four outputs per thread and the loads of up to 8 splits
// issued before the adds (the one-float loop was latency-bound: ~5 us for
// the prefill's 14-22-way splits of 62 x 896).  total % 4 == 0, 16-byte
// aligned ws and Y.
extern "C" __global__ void gemm_splitk_reduce4(const float *__restrict__ ws, float *__restrict__ Y, long total,
                                               int splits) {
    const long n4 = total / 4;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < splits; s0 += 8) {
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; j++)
                v[j] = s0 + j < splits ? __ldcg(reinterpret_cast<const float4 *>(ws + (size_t)(s0 + j) * total) + i)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (s0 + j < splits) {
                    acc.x += v[j].x;
                    acc.y += v[j].y;
                    acc.z += v[j].z;
                    acc.w += v[j].w;
                }
        }
        reinterpret_cast<float4 *>(Y)[i] = acc;
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

// ---------------------------------------------------------------------------
// sgemm_3xtf32_tc: opt-in FP32 SGEMM C = A.B (row-major, the contract of the
// reference's sgemm kernels, switch_gpu.cu:5-39) on the TF32 tensor pipe with
// the 3xTF32 split: each staged operand tile X is read by the tensor pipe as
// big = X with its 13 low mantissa bits ignored (the kind::tf32 operand
// rule: the pipe truncates, so the raw FP32 tile already IS big), and a
// second tile small = X - big (exact in FP32) is written next to it; every
// k-step issues small_A.big_B + big_A.small_B + big_A.big_B into the same
// FP32 TMEM accumulator.  (Writing big back with the bits cleared, as a first
// version did, gave identical results and cost 9-19 % in shared-memory
// traffic.)  The dropped small.small term is ~2^-22 relative, so the
// result is FP32-accurate (relative Frobenius error ~1e-6 against the FP32
// loop) at tensor-pipe speed.
//   * B is first transposed (transpose_f32) into a K-major copy Bt[N][K];
//     reading B's rows directly as an MN-major tf32 operand produced zero
//     products on this part, so both operands use the K-major descriptor;
//   * CTA tile 128 x 128, k-slice 32, 3-stage TMA ring (A box {32 k, 128
//     rows}, Bt box {32 k, 128 rows}), 128-byte swizzle;
//   * warp 0 lane 0 TMA producer; warps 2-5 split each stage (big/small),
//     promote finished accumulators into FP32 registers, and store C;
//     warp 1 lane 0 issues tcgen05.mma kind::tf32 (M=128, N=128, K=8);
//   * M, N arbitrary (TMA zero-fills outside), K % 4 == 0 (16-byte TMA
//     strides) and N % 4 == 0 (vector stores);
//   * with fewer tiles than SMs (short M, e.g. a prompt prefill) the K range
//     is split over `splits` CTAs per tile; each writes its partial tile to
//     ws[split][M][N] and gemm_splitk_reduce adds them in split order.
namespace t3 {
constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3, THREADS = 192;
// The tensor pipe's FP32 accumulation is not IEEE-rounded and its error
// grows with the length of an accumulation chain (measured: one chain over
// K = 2048 gave a relative error of 1.5e-5; 4096-long chains at K = 16384
// gave 2.9e-5).  So every CHUNK k-slices (512 k) the MMAs switch to the
// other of two TMEM accumulators, and the epilogue warps add the finished one
// into FP32 registers with IEEE adds ("promotion"), two slices later, so the
// MMAs never wait for it.
constexpr int NACC = 2, CHUNK = 16;
constexpr int TILE = BM * BK * 4;  // 16 KB: the A tile, the Bt tile, and their small parts
constexpr int STAGE = 4 * TILE;
SB_DEV uint64_t desc_k(const void *p) {  // K-major, 128-byte rows, 8-row atoms 1024 B apart
    return ((tck::smem_u32(p) >> 4) & 0x3fffull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
SB_DEV uint32_t idesc_tf32() {
    return (1u << 4)                             // D f32
           | (2u << 7) | (2u << 10)              // A, B tf32, both K-major
           | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}
SB_DEV void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(
            d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
SB_DEV void mbar_arrive(uint64_t *mb) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tck::smem_u32(mb)) : "memory");
}
}  // namespace t3

// Outputs of the multi-destination form (sgemm_3xtf32_tc_dst): each
// finished row of a tile is stored into every one of them -- this GPU's C
// and the peer ranks' C mapped into this process -- so a row-panel product
// reaches every rank with no separate all-gather.
#define T3_MAX_DST 8
struct T3Dst {
    float *c[T3_MAX_DST];
    int n;
};

// grid: ceil(M/128) * ceil(N/128) * splits CTAs (blockIdx.x = (tile_m *
// tiles_n + tile_n) * splits + split); block t3::THREADS; dynamic smem:
// 1024 + STAGES * STAGE + 256 bytes.  splits == 1: C; else ws[split][M][N].
// MULTI (splits == 1, N % 128 == 0): every matrix of *dst instead of C.
template <bool MULTI>
__device__ __forceinline__ void sgemm3x_body(const CUtensorMap &tm_a, const CUtensorMap &tm_bt, float *__restrict__ C,
                                             int M, int N, int K, float *__restrict__ ws, int splits,
                                             const T3Dst *dst) {
    using namespace t3;
    extern __shared__ __align__(1024) unsigned char smem_raw3[];  // the dynamic shared memory (one name per function)
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw3) + 1023) & ~uintptr_t(1023));
    // stage s: [A | Bt | A small | Bt small], 16 KB each
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE);
    uint64_t *full = bars, *conv = bars + STAGES, *empty = bars + 2 * STAGES;
    uint64_t *acc_full = bars + 3 * STAGES, *acc_empty = acc_full + NACC;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + NACC);
    uint64_t *fin = acc_empty + NACC + 1;  // the MMA issuer's last commit
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + BN - 1) / BN;
    const int tile = blockIdx.x / splits, split = blockIdx.x % splits;
    const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
    const int nk_all = (K + BK - 1) / BK;
    const int kt0 = (int)((long)nk_all * split / splits);
    const int nk = (int)((long)nk_all * (split + 1) / splits) - kt0;  // k-slices of this CTA

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            tck::mbar_init(&full[s], 1);
            tck::mbar_init(&conv[s], 128);
            tck::mbar_init(&empty[s], 1);
        }
        for (int q = 0; q < NACC; q++) {
            tck::mbar_init(&acc_full[q], 1);
            tck::mbar_init(&acc_empty[q], 128);
        }
        tck::mbar_init(fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tck::smem_u32(tmem_slot)),
                     "r"(BN * NACC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            int issued = 0;
            for (int kt = 0; kt < nk; kt++, issued++) {
                const int s = kt % STAGES;
                if (kt >= STAGES && !tck::mbar_wait(&empty[s], ((kt / STAGES) - 1) & 1)) break;
                unsigned char *st = smem + (size_t)s * STAGE;
                tck::mbar_expect_tx(&full[s], 2 * TILE);
                tck::tma_2d(st, &tm_a, (kt0 + kt) * BK, m0, &full[s]);
                tck::tma_2d(st + TILE, &tm_bt, (kt0 + kt) * BK, n0, &full[s]);
            }
            for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; i++)
                tck::mbar_wait(&full[i % STAGES], (i / STAGES) & 1, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            const uint32_t idesc = idesc_tf32();
            for (int kt = 0; kt < nk; kt++) {
                const int s = kt % STAGES, c = kt / CHUNK, q = c % NACC;
                // a chunk's accumulator is reused once the chunk NACC before it was promoted
                if (kt % CHUNK == 0 && c >= NACC && !tck::mbar_wait(&acc_empty[q], ((c / NACC) - 1) & 1)) break;
                if (!tck::mbar_wait(&conv[s], (kt / STAGES) & 1)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                unsigned char *st = smem + (size_t)s * STAGE;
                const uint64_t a = desc_k(st), b = desc_k(st + TILE), as = desc_k(st + 2 * TILE), bs = desc_k(st + 3 * TILE);
                const uint32_t d = tmem + (uint32_t)(q * BN);
#pragma unroll
                for (int k = 0; k < BK / 8; k++) {
                    const uint64_t dk = 2ull * k;  // +32 B per K=8 step inside the swizzled 128-byte rows
                    mma_tf32(d, as + dk, b + dk, idesc, (kt % CHUNK > 0 || k > 0) ? 1u : 0u);
                    mma_tf32(d, a + dk, bs + dk, idesc, 1u);
                    mma_tf32(d, a + dk, b + dk, idesc, 1u);
                }
                tck::mma_commit(&empty[s]);
                if (kt % CHUNK == CHUNK - 1 || kt == nk - 1) tck::mma_commit(&acc_full[q]);
            }
            // no MMA may still write tensor memory when it is freed below
            tck::mma_commit(fin);
            tck::mbar_wait(fin, 0, false);
        }
    } else {
        // ---- warps 2-5: split each stage into big/small, promote finished
        // accumulators into FP32 registers, then store C
        const int ct = threadIdx.x - 64;  // 0..127
        const int quarter = warp & 3;      // TMEM lanes 32*quarter.. belong to this warp
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        const int nchunks = (nk + CHUNK - 1) / CHUNK;
        float sum[BN];
#pragma unroll
        for (int j = 0; j < BN; j++) sum[j] = 0.f;
        bool ok = true;
        int promoted = 0;
        auto promote = [&](int c) {  // add chunk c's accumulator into sum, release it
            const int q = c % NACC;
            ok = ok && tck::mbar_wait(&acc_full[q], (c / NACC) & 1);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int col = 0; col < BN; col += 16) {
                float v[16];
                tck::tmem_ld16(lane_base + (uint32_t)(q * BN + col), v);
#pragma unroll
                for (int j = 0; j < 16; j++) sum[col + j] += v[j];
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            t3::mbar_arrive(&acc_empty[q]);
        };
        for (int kt = 0; kt < nk && ok; kt++) {
            const int s = kt % STAGES;
            ok = tck::mbar_wait(&full[s], (kt / STAGES) & 1);
            if (!ok) break;
            unsigned char *st = smem + (size_t)s * STAGE;
#pragma unroll
            for (int half = 0; half < 2; half++) {  // A tile, then Bt tile
                uint4 *src = reinterpret_cast<uint4 *>(st + half * TILE);
                uint4 *dst = reinterpret_cast<uint4 *>(st + (2 + half) * TILE);
#pragma unroll 4
                for (int i = ct; i < TILE / 16; i += 128) {
                    uint4 v = src[i], big, small;
                    big.x = v.x & 0xFFFFE000u; big.y = v.y & 0xFFFFE000u;
                    big.z = v.z & 0xFFFFE000u; big.w = v.w & 0xFFFFE000u;
                    small.x = __float_as_uint(__uint_as_float(v.x) - __uint_as_float(big.x));
                    small.y = __float_as_uint(__uint_as_float(v.y) - __uint_as_float(big.y));
                    small.z = __float_as_uint(__uint_as_float(v.z) - __uint_as_float(big.z));
                    small.w = __float_as_uint(__uint_as_float(v.w) - __uint_as_float(big.w));
                    dst[i] = small;  // big stays in place: see the note above the kernel
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
            mbar_arrive(&conv[s]);
            // chunk c is promoted two slices after it ended, when its MMAs have drained
            if (kt >= CHUNK + 1 && (kt - 1) % CHUNK == 0) promote(promoted++);
        }
        while (ok && promoted < nchunks) promote(promoted++);
        const int row = m0 + quarter * 32 + lane;
        if (MULTI) {
            // this warp's 32 rows through the drained stage buffers (rows
            // 132 floats apart: each float4 store of the warp hits every
            // bank once per 8 lanes), then whole 512-byte row segments to
            // every destination -- full lines over NVLink
            float *st = reinterpret_cast<float *>(smem) + (size_t)quarter * 32 * 132;
#pragma unroll
            for (int j = 0; j < BN; j += 4)
                *reinterpret_cast<float4 *>(st + lane * 132 + j) = make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
            __syncwarp();
            if (__all_sync(0xffffffffu, ok)) {
                for (int r = 0; r < 32; r++) {
                    const float4 v = *reinterpret_cast<const float4 *>(st + r * 132 + lane * 4);
                    const size_t off = (size_t)(m0 + quarter * 32 + r) * N + n0 + lane * 4;
                    if (m0 + quarter * 32 + r < M)
                        for (int d = 0; d < dst->n; d++) *reinterpret_cast<float4 *>(dst->c[d] + off) = v;
                }
            }
        } else if (ok && row < M) {
            float *crow = (splits == 1 ? C : ws + (size_t)split * M * N) + (size_t)row * N + n0;
            if (n0 + BN <= N) {
#pragma unroll
                for (int j = 0; j < BN; j += 4) *reinterpret_cast<float4 *>(crow + j) = make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < BN; j++)
                    if (n0 + j < N) crow[j] = sum[j];
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(BN * NACC))
                     : "memory");
    }
}

extern "C" __global__ void __launch_bounds__(t3::THREADS, 1)
    sgemm_3xtf32_tc(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_bt,
                    float *__restrict__ C, int M, int N, int K, float *__restrict__ ws, int splits) {
    sgemm3x_body<false>(tm_a, tm_bt, C, M, N, K, ws, splits, nullptr);
}

// The multi-destination form (splits == 1; M, N % 128 == 0): plain stores
// to local or peer-mapped outputs (never TMA), and a system-scope fence so
// the peers see them once the kernel completes.
extern "C" __global__ void __launch_bounds__(t3::THREADS, 1)
    sgemm_3xtf32_tc_dst(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_bt,
                        const __grid_constant__ T3Dst dst, int M, int N, int K) {
    sgemm3x_body<true>(tm_a, tm_bt, nullptr, M, N, K, nullptr, 1, &dst);
    __threadfence_system();
}

// out[c][r] = in[r][c] for a rows x cols FP32 matrix (32 x 32 tiles through
// shared memory, both sides coalesced); grid (ceil(cols/32), ceil(rows/32)),
// block 256 (1-D: tx = thread % 32, ty = thread / 32 in 0..7).
extern "C" __global__ void __launch_bounds__(256) transpose_f32(const float *__restrict__ in, float *__restrict__ out,
                                                               int rows, int cols) {
    __shared__ float t[32][33];
    if (blockDim.x != 256) return;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + tx;
        if (r < rows && c < cols) t[i][tx] = in[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + tx;
        if (c < cols && r < rows) out[(size_t)c * rows + r] = t[tx][i];
    }
}

// ---------------------------------------------------------------------------
// sgemm_tma: the FP32 CUDA-core SGEMM (C = A.B row-major, the contract of the
// reference's sgemm kernels, switch_gpu.cu:5-39) with its operand tiles
// staged by TMA instead of by the threads:
//   * persistent CTAs (one per SM), 288 threads: warp 8 lane 0 is the TMA
//     producer, warps 0-7 (256 threads) compute 128 x 128 tiles, 8 x 8
//     outputs per thread as packed fma.rn.f32x2;
//   * a 4-stage ring of 32-deep k-slices: A box {32 k, 128 rows} with the
//     128-byte swizzle (rows 128 B: chunk c of row r lands at c ^ (r & 7)),
//     B box {128 n, 32 k} dense; full[s] mbarriers with transaction counts,
//     empty[s] released by one lane of each compute warp;
//   * a thread owns rows ty + 16 i (i < 8) -- so the four ty of a warp hit
//     four different swizzled chunks (no bank conflicts) -- and columns
//     tx * 4 .. + 3 and 64 + tx * 4 .. + 3; it reads A four k at a time
//     (one 128-bit load per row) and B one k-row at a time;
//   * every output is one fma.rn chain over k in order, as in sgemm_b200, so
//     the two kernels give bit-identical results; TMA zero-fills outside
//     the matrices (any M, N; K % 4 == 0 and N % 4 == 0 for the 16-byte
//     strides).
// The threads no longer load, transpose and store the tiles, so their issue
// slots go to the FMAs.
namespace sgt {
constexpr int BM = 128, BN = 128, BK = 32, STAGES = 4, THREADS = 288;
constexpr int A_BYTES = BM * BK * 4, B_BYTES = BK * BN * 4, STAGE = A_BYTES + B_BYTES;
SB_DEV void mbar_arrive(uint64_t *mb) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tck::smem_u32(mb)) : "memory");
}
}  // namespace sgt

// grid: min(tiles, SMs) CTAs, or in stream-K mode (ws != null; M, N % 128 ==
// 0, K % 32 == 0) G > tiles CTAs; block sgt::THREADS; dynamic smem 1024 +
// STAGES * STAGE + 128.
extern "C" __global__ void __launch_bounds__(sgt::THREADS, 1)
    sgemm_tma(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, float *__restrict__ C,
              int M, int N, int K, float *__restrict__ ws) {
    using namespace sgt;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE), *empty = full + STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN, ntiles = tiles_m * tiles_n;
    const int nk = (K + BK - 1) / BK;
    // work items: whole tiles (ws == nullptr), or stream-K pieces -- the
    // tiles x nk k-slices cut into gridDim.x equal ranges, one per CTA; a
    // piece (one tile's slices within the range) goes to ws[2 * cta +
    // piece] as a compact 128 x 128 tile for sgemm_stk_fixup to add up
    const bool stk = ws != nullptr;
    const long units = (long)ntiles * nk, u_end = units * (blockIdx.x + 1) / gridDim.x;
    struct Item {
        int tile, k0, k1;
    };
    auto next_item = [&](int item, long &u, Item &it) -> bool {
        if (!stk) {
            it.tile = blockIdx.x + item * gridDim.x;
            it.k0 = 0;
            it.k1 = nk;
            return it.tile < ntiles;
        }
        if (u >= u_end) return false;
        it.tile = (int)(u / nk);
        it.k0 = (int)(u % nk);
        it.k1 = (int)min((long)nk, u_end - (long)it.tile * nk);
        u = (long)it.tile * nk + it.k1;
        return true;
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            tck::mbar_init(&full[s], 1);
            tck::mbar_init(&empty[s], 8);  // one lane of each compute warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // grouped raster (8 tile-rows share B's column panels in L2), as sgemm_b200
    auto tile_mn = [=](int tile) {
        const int per_group = 8 * tiles_n, first_m = (tile / per_group) * 8;
        const int gsz = min(tiles_m - first_m, 8);
        return make_int2((first_m + (tile % per_group) % gsz) * BM, ((tile % per_group) / gsz) * BN);
    };
    if (warp == 8) {
        if (lane == 0) {  // ---- TMA producer
            long it = 0, u = units * blockIdx.x / gridDim.x;
            bool ok = true;
            Item w;
            for (int item = 0; ok && next_item(item, u, w); item++) {
                const int2 mn = tile_mn(w.tile);
                const int m0 = mn.x, n0 = mn.y;
                for (int kt = w.k0; kt < w.k1; kt++, it++) {
                    const int s = (int)(it % STAGES);
                    if (it >= STAGES && !(ok = tck::mbar_wait(&empty[s], (unsigned)(((it / STAGES) - 1) & 1)))) break;
                    unsigned char *st = smem + (size_t)s * STAGE;
                    tck::mbar_expect_tx(&full[s], STAGE);
                    tck::tma_2d(st, &tm_a, kt * BK, m0, &full[s]);
                    tck::tma_2d(st + A_BYTES, &tm_b, n0, kt * BK, &full[s]);
                }
            }
            // every stage issued must have landed before this CTA may exit
            for (long i = (it > STAGES ? it - STAGES : 0); i < it; i++)
                tck::mbar_wait(&full[i % STAGES], (unsigned)((i / STAGES) & 1), false);
        }
        return;
    }
    // ---- warps 0-7: compute
    const int ty = (warp >> 1) * 4 + (lane >> 3);  // 0..15
    const int tx = (warp & 1) * 8 + (lane & 7);    // 0..15
    long it = 0, u = units * blockIdx.x / gridDim.x;
    bool ok = true;
    Item w;
    for (int item = 0; ok && next_item(item, u, w); item++) {
        const int2 mn = tile_mn(w.tile);
        const int m0 = mn.x, n0 = mn.y;
        unsigned long long acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0ull;
        for (int kt = w.k0; kt < w.k1; kt++, it++) {
            const int s = (int)(it % STAGES);
            if (!(ok = tck::mbar_wait(&full[s], (unsigned)((it / STAGES) & 1)))) break;
            const float *As = reinterpret_cast<const float *>(smem + (size_t)s * STAGE);
            const float *Bs = reinterpret_cast<const float *>(smem + (size_t)s * STAGE + A_BYTES);
#pragma unroll 1
            for (int kq = 0; kq < BK / 4; kq++) {
                float4 a[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int r = ty + 16 * i;
                    a[i] = *reinterpret_cast<const float4 *>(As + r * BK + ((kq ^ (r & 7)) << 2));
                }
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    const float *brow = Bs + (kq * 4 + kk) * BN;
                    const float4 b0 = *reinterpret_cast<const float4 *>(brow + tx * 4);
                    const float4 b1 = *reinterpret_cast<const float4 *>(brow + 64 + tx * 4);
                    const unsigned long long bp[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y),
                                                      f2_pack(b1.z, b1.w)};
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float av = reinterpret_cast<const float *>(&a[i])[kk];
                        const unsigned long long ai = f2_pack(av, av);
#pragma unroll
                        for (int j = 0; j < 4; j++) acc[i][j] = ffma2(ai, bp[j], acc[i][j]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) sgt::mbar_arrive(&empty[s]);  // this warp is done with the stage
        }
        if (!ok) break;
        if (stk) {  // the piece, compact, to its workspace slot
            float *pw = ws + (size_t)(2 * blockIdx.x + item) * BM * BN;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int hb = 0; hb < 2; hb++) {
                    float4 o;
                    f2_unpack(acc[i][hb * 2], o.x, o.y);
                    f2_unpack(acc[i][hb * 2 + 1], o.z, o.w);
                    *reinterpret_cast<float4 *>(pw + (ty + 16 * i) * BN + hb * 64 + tx * 4) = o;
                }
            continue;
        }
        // epilogue: rows ty + 16 i, columns tx * 4 and 64 + tx * 4 (4 each)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = m0 + ty + 16 * i;
            if (r >= M) continue;
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
                const int c = n0 + hb * 64 + tx * 4;
                float4 o;
                f2_unpack(acc[i][hb * 2], o.x, o.y);
                f2_unpack(acc[i][hb * 2 + 1], o.z, o.w);
                float *p = C + (size_t)r * N + c;
                if (c + 3 < N) {
                    *reinterpret_cast<float4 *>(p) = o;
                } else {
                    if (c + 0 < N) p[0] = o.x;
                    if (c + 1 < N) p[1] = o.y;
                    if (c + 2 < N) p[2] = o.z;
                }
            }
        }
    }
}
