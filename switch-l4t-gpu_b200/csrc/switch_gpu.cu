// switch_gpu.cu -- the "switch_gpu" module image (sm_100a cubin): the SGEMM
// family and the bandwidth probe with the reference's names and parameter
// lists (switch_gpu.cu of pkia/switch-l4t-gpu), plus this package's own
// entry points.
//
// SGEMM design (FP32 CUDA cores; B200 has no FP32 tensor path):
//   * 128x128 CTA tile, 16-deep k-slices, 256 threads, 8x8 outputs per
//     thread as 2x2 blocks of 4x4 (rows ty*4 and 64+ty*4, cols tx*4 and
//     64+tx*4).  A warp covers 4 (ty) x 8 (tx) threads, so each 128-bit
//     fragment load from shared memory touches 4 or 8 distinct 16-byte words:
//     one wavefront, broadcast to the other lanes.
//   * Packed FP32 FMA (fma.rn.f32x2): each instruction updates two adjacent
//     columns of one output row, so the 64 FMAs of a k-step issue as 32
//     instructions and the issue slots left over hide the fragment loads.
//     Every output is still one fma.rn chain over k in order, so results are
//     bit-identical to a scalar fmaf loop.
//   * 128 registers per thread: two CTAs (16 warps) per SM, so one CTA's
//     barrier and tile prologue overlap the other's FMAs.
//   * A is stored k-major (transposed) in shared memory; its 16-byte units
//     are XOR-swizzled by k (unit ^ 4*(k/4)) so the transposing 32-bit stores
//     of a warp (16 rows x 2 k-quads) hit 32 distinct banks while fragment
//     reads stay 128-bit.  B is stored as loaded.  Two shared buffers: the
//     next k-slice is fetched into registers (two float4 of A and two of B
//     per thread) while the current one is multiplied, then stored into the
//     other buffer -- one __syncthreads per 16 k (a 16-deep slice measured
//     4-5 % faster than 8-deep: half the barriers).
//   * Tiles are walked by a grid-stride loop over a grouped (8 tile-rows)
//     order, so ANY grid shape is correct -- the stock harness launches
//     (n/32)^2 or (n/64)^2 CTAs of 16x16 threads (gpu_workload.c:90,142,168)
//     and no dynamic shared memory (the 32 KB here are static).  This
//     package launches one CTA per tile.
//   * Shapes that are multiples of the tile (M, N of 128, K of 16) with
//     16-byte aligned pointers take unpredicated 128-bit loads and stores;
//     anything else takes the same loop with zero-filled predicated scalar
//     loads and guarded stores.
#include "sb_common.cuh"

#define SG_BM 128
#define SG_BN 128
#define SG_BK 16
#define SG_THREADS 256

struct SgSmem {
    float As[2][SG_BK][SG_BM];  // k-major, 16-byte units swizzled by sg_swz(k)
    float Bs[2][SG_BK][SG_BN];
};
// Output matrices of the multi-destination form (sgemm_b200_dst): every
// finished tile is stored into each of them -- this GPU's C and the C of
// each peer rank, mapped into this process -- so the row panels of all
// ranks meet in every rank's C with no separate all-gather.
#define SG_MAX_DST 8
struct SgDst {
    float *c[SG_MAX_DST];
    int n;
};
__device__ __forceinline__ int sg_swz(int k) { return (k >> 2) << 2; }

// One k-slice into registers with zero fill outside the matrices: A row
// m0+ar, k-quad k0+ak; B k-row k0+br, columns n0+bc..+3.
__device__ __forceinline__ void sg_load_slice(const float *__restrict__ A, const float *__restrict__ B, int M,
                                              int N, int K, int m0, int n0, int k0, int ar, int ak, int br, int bc,
                                              float4 &ra, float4 &rb) {
    const int r = m0 + ar, c = k0 + ak;
    const float *pa = A + (size_t)r * K;
    ra.x = (r < M && c + 0 < K) ? pa[c + 0] : 0.f;
    ra.y = (r < M && c + 1 < K) ? pa[c + 1] : 0.f;
    ra.z = (r < M && c + 2 < K) ? pa[c + 2] : 0.f;
    ra.w = (r < M && c + 3 < K) ? pa[c + 3] : 0.f;
    const int kr = k0 + br, n = n0 + bc;
    const float *pb = B + (size_t)kr * N;
    rb.x = (kr < K && n + 0 < N) ? pb[n + 0] : 0.f;
    rb.y = (kr < K && n + 1 < N) ? pb[n + 1] : 0.f;
    rb.z = (kr < K && n + 2 < N) ? pb[n + 2] : 0.f;
    rb.w = (kr < K && n + 3 < N) ? pb[n + 3] : 0.f;
}

__device__ __forceinline__ void sg_store_slice(SgSmem &s, int buf, int ams, int ak, int br, int bc, const float4 &ra,
                                               const float4 &rb) {
    s.As[buf][ak + 0][ams] = ra.x;
    s.As[buf][ak + 1][ams] = ra.y;
    s.As[buf][ak + 2][ams] = ra.z;
    s.As[buf][ak + 3][ams] = ra.w;
    *reinterpret_cast<float4 *>(&s.Bs[buf][br][bc]) = rb;
}

// 64 rows x 128 columns staged in shared memory -> rows r0.., columns n0..
// of C (or of every destination): each warp stores whole 512-byte row
// segments.  Not inlined, so the stores' registers never weigh on the main
// loop's.  (With the 8 x 8 register tile written straight from the
// registers, the kernel kept more spills in its loop and took 3 % longer
// at 8192 x 16384 x 16384.)
__device__ __noinline__ void sg_copy_out1(const float *st, float *C, int r0, int n0, int N, int tid) {
    for (int k = tid; k < 64 * SG_BN / 4; k += SG_THREADS) {
        const int row = k / (SG_BN / 4), c4 = k % (SG_BN / 4);
        *reinterpret_cast<float4 *>(C + (size_t)(r0 + row) * N + n0 + c4 * 4) =
            *reinterpret_cast<const float4 *>(st + row * SG_BN + c4 * 4);
    }
}
__device__ __noinline__ void sg_copy_out(const float *st, const SgDst *dst, int r0, int n0, int N, int tid) {
    for (int k = tid; k < 64 * SG_BN / 4; k += SG_THREADS) {
        const int row = k / (SG_BN / 4), c4 = k % (SG_BN / 4);
        const float4 v = *reinterpret_cast<const float4 *>(st + row * SG_BN + c4 * 4);
        const size_t off = (size_t)(r0 + row) * N + n0 + c4 * 4;
        for (int d = 0; d < dst->n; d++) *reinterpret_cast<float4 *>(dst->c[d] + off) = v;
    }
}

// k range [kbeg, kbeg + klen) of the product (split-K: the unpredicated
// path only, kbeg and klen multiples of SG_BK); K stays A's row stride.
// LOCAL: the tile is written to C as a compact 128 x 128 block (a piece of
// a tile in the stream-K form) instead of at its place in the M x N matrix.
// MULTI (unpredicated path only): the tile goes to every matrix of *dst
// instead of C.
template <bool EDGE, bool LOCAL = false, bool MULTI = false>
__device__ __forceinline__ void sgemm_tiles(const float *__restrict__ A, const float *__restrict__ B,
                                            float *__restrict__ C, int M, int N, int K, int tid, int cta,
                                            int ncta, SgSmem &s, int kbeg = 0, int klen = -1,
                                            const SgDst *dst = nullptr) {
    if (klen < 0) klen = K;
    const int warp = tid >> 5, lane = tid & 31;
    const int ty = (warp >> 1) * 4 + (lane >> 3);  // 0..15
    const int tx = (warp & 1) * 8 + (lane & 7);    // 0..15
    const int ar = tid >> 1, ak = (tid & 1) * 4;   // A loader: row, k-quad
    const int br = tid >> 5, bc = (tid & 31) * 4;  // B loader: k-row, column quad
    const int ams = (((ar >> 2) ^ sg_swz(ak)) << 2) | (ar & 3);
    const int ams2 = (((ar >> 2) ^ sg_swz(ak + 8)) << 2) | (ar & 3);
    const int tiles_m = (M + SG_BM - 1) / SG_BM, tiles_n = (N + SG_BN - 1) / SG_BN;
    const int ntiles = tiles_m * tiles_n;
    const int nk = (klen + SG_BK - 1) / SG_BK;

    for (int tile = cta; tile < ntiles; tile += ncta) {
        // grouped raster: 8 tile-rows share the B column panels in L2
        const int per_group = 8 * tiles_n;
        const int first_m = (tile / per_group) * 8;
        const int gsz = min(tiles_m - first_m, 8);
        const int tm = first_m + (tile % per_group) % gsz;
        const int tn = (tile % per_group) / gsz;
        const int m0 = tm * SG_BM, n0 = tn * SG_BN;

        unsigned long long acc[8][4];  // (row i, column pair j) as packed f32x2
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = 0ull;

        // unpredicated path: running pointers to this thread's A row / B k-row
        const float *Ap = A + (size_t)(m0 + ar) * K + kbeg + ak;
        const float *Bp = B + (size_t)(kbeg + br) * N + n0 + bc;
        float4 ra, rb, ra2, rb2;
        if (EDGE) {
            sg_load_slice(A, B, M, N, K, m0, n0, 0, ar, ak, br, bc, ra, rb);
            sg_load_slice(A, B, M, N, K, m0, n0, 0, ar, ak + 8, br + 8, bc, ra2, rb2);
        } else {
            ra = __ldg(reinterpret_cast<const float4 *>(Ap));
            rb = __ldg(reinterpret_cast<const float4 *>(Bp));
            ra2 = __ldg(reinterpret_cast<const float4 *>(Ap + 8));
            rb2 = __ldg(reinterpret_cast<const float4 *>(Bp + (size_t)8 * N));
        }
        __syncthreads();  // previous tile's readers are done with buffer 0
        sg_store_slice(s, 0, ams, ak, br, bc, ra, rb);
        sg_store_slice(s, 0, ams2, ak + 8, br + 8, bc, ra2, rb2);
        __syncthreads();
        for (int kt = 0; kt < nk; kt++) {
            const int buf = kt & 1;
            if (kt + 1 < nk) {
                if (EDGE) {
                    sg_load_slice(A, B, M, N, K, m0, n0, (kt + 1) * SG_BK, ar, ak, br, bc, ra, rb);
                    sg_load_slice(A, B, M, N, K, m0, n0, (kt + 1) * SG_BK, ar, ak + 8, br + 8, bc, ra2, rb2);
                } else {
                    Ap += SG_BK;
                    Bp += (size_t)SG_BK * N;
                    ra = __ldg(reinterpret_cast<const float4 *>(Ap));
                    rb = __ldg(reinterpret_cast<const float4 *>(Bp));
                    ra2 = __ldg(reinterpret_cast<const float4 *>(Ap + 8));
                    rb2 = __ldg(reinterpret_cast<const float4 *>(Bp + (size_t)8 * N));
                }
            }
#pragma unroll
            for (int k = 0; k < SG_BK; k++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&s.As[buf][k][(ty ^ sg_swz(k)) * 4]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&s.As[buf][k][((16 + ty) ^ sg_swz(k)) * 4]);
                const float4 b0 = *reinterpret_cast<const float4 *>(&s.Bs[buf][k][tx * 4]);
                const float4 b1 = *reinterpret_cast<const float4 *>(&s.Bs[buf][k][64 + tx * 4]);
                const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const unsigned long long bp[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y),
                                                  f2_pack(b1.z, b1.w)};
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const unsigned long long ai = f2_pack(a[i], a[i]);
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = ffma2(ai, bp[j], acc[i][j]);
                }
            }
            if (kt + 1 < nk) {
                sg_store_slice(s, buf ^ 1, ams, ak, br, bc, ra, rb);
                sg_store_slice(s, buf ^ 1, ams2, ak + 8, br + 8, bc, ra2, rb2);
            }
            __syncthreads();
        }
        if (!EDGE && !LOCAL) {
            // whole tiles: through shared memory, 64 rows at a time, stored
            // as whole 512-byte row segments to C (or every destination)
            float *st = reinterpret_cast<float *>(&s);  // 8192 floats: one half-tile
#pragma unroll
            for (int h = 0; h < 2; h++) {
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int hb = 0; hb < 2; hb++) {
                        float4 o;
                        f2_unpack(acc[4 * h + i][hb * 2], o.x, o.y);
                        f2_unpack(acc[4 * h + i][hb * 2 + 1], o.z, o.w);
                        *reinterpret_cast<float4 *>(st + (ty * 4 + i) * SG_BN + hb * 64 + tx * 4) = o;
                    }
                __syncthreads();
                if (MULTI) sg_copy_out(st, dst, m0 + 64 * h, n0, N, tid);
                else sg_copy_out1(st, C, m0 + 64 * h, n0, N, tid);
                __syncthreads();  // the half is read before the next one (or the next tile) overwrites it
            }
        } else {
        // epilogue of partial tiles and stream-K pieces: straight from the registers
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = m0 + (i >> 2) * 64 + ty * 4 + (i & 3);
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
                const int c = n0 + hb * 64 + tx * 4;
                float4 o;
                f2_unpack(acc[i][hb * 2], o.x, o.y);
                f2_unpack(acc[i][hb * 2 + 1], o.z, o.w);
                float *p = LOCAL ? C + (size_t)(r - m0) * SG_BN + (c - n0) : C + (size_t)r * N + c;
                if (!EDGE) {
                    *reinterpret_cast<float4 *>(p) = o;
                } else if (r < M) {
                    if (c + 0 < N) p[0] = o.x;
                    if (c + 1 < N) p[1] = o.y;
                    if (c + 2 < N) p[2] = o.z;
                    if (c + 3 < N) p[3] = o.w;
                }
            }
        }
        }
    }
}

// Any-shape fallback for launches whose block is not 256 threads: each
// thread computes whole outputs.
__device__ __noinline__ void sgemm_any(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C, int M,
                          int N, int K) {
    const long nthreads = (long)gridDim.x * gridDim.y * gridDim.z * blockDim.x * blockDim.y * blockDim.z;
    const long cta = (blockIdx.z * gridDim.y + blockIdx.y) * (long)gridDim.x + blockIdx.x;
    const long tid = cta * blockDim.x * blockDim.y * blockDim.z +
                     (threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x;
    for (long o = tid; o < (long)M * N; o += nthreads) {
        const int i = (int)(o / N), j = (int)(o % N);
        float acc = 0.0f;
        for (int k = 0; k < K; k++) acc = fmaf(A[(size_t)i * K + k], B[(size_t)k * N + j], acc);
        C[o] = acc;
    }
}

// The predicated path as its own (not inlined) function, so its extra
// registers do not constrain the allocation of the unpredicated loop.
__device__ __noinline__ void sgemm_edge(const float *A, const float *B, float *C, int M, int N, int K, int tid,
                                        int cta, int ncta, SgSmem &s) {
    sgemm_tiles<true>(A, B, C, M, N, K, tid, cta, ncta, s);
}

__device__ __forceinline__ void sgemm_entry(const float *A, const float *B, float *C, int M, int N, int K) {
    const int nth = blockDim.x * blockDim.y * blockDim.z;
    if (nth != SG_THREADS) { sgemm_any(A, B, C, M, N, K); return; }
    const int tid = (threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x;
    const int cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const int ncta = gridDim.x * gridDim.y * gridDim.z;
    const bool whole = (M % SG_BM) == 0 && (N % SG_BN) == 0 && (K % SG_BK) == 0 &&
                       ((((uintptr_t)A) | ((uintptr_t)B) | ((uintptr_t)C)) & 15) == 0;
    __shared__ __align__(16) SgSmem s;
    if (whole) sgemm_tiles<false>(A, B, C, M, N, K, tid, cta, ncta, s);
    else sgemm_edge(A, B, C, M, N, K, tid, cta, ncta, s);
}

// Reference: switch_gpu.cu:5-39 (stock launch: grid (n/32, n/32), block 16x16).
extern "C" __global__ void __launch_bounds__(256, 2)
    sgemm_tiled(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C, int M, int N, int K) {
    sgemm_entry(A, B, C, M, N, K);
}
// Reference: switch_gpu.cu:59-95 (stock launch: grid (n/64, n/64), block 16x16).
extern "C" __global__ void __launch_bounds__(256, 2)
    sgemm_tiled4(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C, int M, int N, int K) {
    sgemm_entry(A, B, C, M, N, K);
}
// Reference: switch_gpu.cu:99-137 (stock launch: grid (n/64, n/64), block 16x16).
extern "C" __global__ void __launch_bounds__(256, 2)
    sgemm_opt(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C, int M, int N, int K) {
    sgemm_entry(A, B, C, M, N, K);
}
// This package's launch of the same kernel body: one CTA per 128x128 tile,
// block 256 (issued by sb_sgemm).
extern "C" __global__ void __launch_bounds__(256, 2)
    sgemm_b200(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C, int M, int N, int K) {
    sgemm_entry(A, B, C, M, N, K);
}

// The multi-destination form: C = A.B for whole tiles (M, N % 128 == 0,
// K % 16 == 0, 16-byte aligned), each tile stored into every matrix of
// dst -- up to SG_MAX_DST, local or peer-mapped over NVLink (plain stores,
// no TMA).  The system-scope fence at the end makes this CTA's remote
// stores visible to the peers before the kernel completes; the caller
// orders their readers after the kernel (a collective, an event).
// One CTA per tile, block 256.
extern "C" __global__ void __launch_bounds__(256, 2)
    sgemm_b200_dst(const float *__restrict__ A, const float *__restrict__ B, const __grid_constant__ SgDst dst,
                   int M, int N, int K) {
    if (blockDim.x * blockDim.y * blockDim.z != SG_THREADS) return;
    __shared__ __align__(16) SgSmem s;
    sgemm_tiles<false, false, true>(A, B, nullptr, M, N, K, threadIdx.x, blockIdx.x, gridDim.x, s, 0, -1, &dst);
    __threadfence_system();
}

// Stream-K form for products with fewer 128 x 128 tiles than two per SM
// (1024^3: 64 tiles): the tiles x K/16 k-chunks of the product are cut into
// gridDim.x equal contiguous ranges, one per CTA (two per SM), so every SM
// gets the same work -- a split-K form (4 k-ranges per tile, partials added
// by a second kernel) left 40 of 148 SMs with one CTA and the rest with two.  A range covers at most two tiles (it is shorter
// than one tile's K); each piece goes to ws[2 * cta + piece] (a compact
// 128 x 128 tile), and sgemm_stk_fixup adds a tile's pieces in CTA order
// (deterministic) into C.
// Needs M, N % 128 == 0, K % 16 == 0, tiles < gridDim.x and 16-byte aligned
// pointers (the host checks).  Block 256.
__device__ __forceinline__ long stk_first(long units, int g, int c) { return units * c / g; }
// the CTA whose range holds unit u: the largest c with units * c / g <= u
__device__ __forceinline__ int stk_owner(long units, int g, long u) { return (int)(((u + 1) * g - 1) / units); }
extern "C" __global__ void __launch_bounds__(256, 2)
    sgemm_b200_stk(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C,
                   float *__restrict__ ws, int M, int N, int K) {
    if (blockDim.x * blockDim.y * blockDim.z != SG_THREADS) return;
    __shared__ __align__(16) SgSmem s;
    const int tiles = (M / SG_BM) * (N / SG_BN), nk = K / SG_BK, G = gridDim.x, cta = blockIdx.x;
    const long units = (long)tiles * nk, u1 = stk_first(units, G, cta + 1);
    int piece = 0;
    for (long u = stk_first(units, G, cta); u < u1; piece++) {
        const int t = (int)(u / nk), k0 = (int)(u % nk);
        const int k1 = (int)min((long)nk, u1 - (long)t * nk);
        sgemm_tiles<false, true>(A, B, ws + (size_t)(2 * cta + piece) * SG_BM * SG_BN, M, N, K, threadIdx.x, t,
                                 tiles, s, k0 * SG_BK, (k1 - k0) * SG_BK);
        u = (long)t * nk + k1;
    }
}
// C tile t = the sum, in CTA order, of its pieces in ws.  One float4 of the
// tile per thread, the loads of up to 8 pieces issued before the adds (a
// loop of dependent piece loads ran at 1.4 TB/s from L2).  grid: tiles x
// 16; block 256; G = the stream-K kernel's grid, bk its k-slice depth (16
// for sgemm_b200_stk, 32 for sgemm_tma).
extern "C" __global__ void __launch_bounds__(256) sgemm_stk_fixup(const float *__restrict__ ws, float *__restrict__ C,
                                                                  int M, int N, int K, int G, int bk) {
    const int tiles_n = N / SG_BN, tiles = (M / SG_BM) * tiles_n, nk = K / bk;
    const int t = blockIdx.x / 16, i = (blockIdx.x % 16) * 256 + threadIdx.x;  // float4 index in the tile
    if (t >= tiles) return;
    const long units = (long)tiles * nk, ub = (long)t * nk, ue = ub + nk;
    const int c_lo = stk_owner(units, G, ub), c_hi = stk_owner(units, G, ue - 1);
    // the tile's row / column in sgemm_tiles' grouped raster
    const int tiles_m = M / SG_BM, per_group = 8 * tiles_n, first_m = (t / per_group) * 8;
    const int gsz = min(tiles_m - first_m, 8);
    const int m0 = (first_m + (t % per_group) % gsz) * SG_BM, n0 = ((t % per_group) / gsz) * SG_BN;
    // every CTA after c_lo starts inside this tile (its piece 0); c_lo's piece
    // is its second one when it started in an earlier tile
    const int lo_piece = stk_first(units, G, c_lo) < ub ? 1 : 0;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = c_lo; c0 <= c_hi; c0 += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = c0 + j;
            v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c <= c_hi) {
                const int piece = c == c_lo ? lo_piece : 0;
                v[j] = __ldcg(reinterpret_cast<const float4 *>(ws + (size_t)(2 * c + piece) * SG_BM * SG_BN) + i);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (c0 + j <= c_hi) {
                acc.x += v[j].x;
                acc.y += v[j].y;
                acc.z += v[j].z;
                acc.w += v[j].w;
            }
    }
    const int r = (i * 4) / SG_BN, col = (i * 4) % SG_BN;
    *reinterpret_cast<float4 *>(C + (size_t)(m0 + r) * N + n0 + col) = acc;
}

// One output per thread, k in order, product and sum rounded separately:
// the same float arithmetic as the harness's CPU loop (gpu_workload.c:97-98),
// so its result is bit-identical to it.  Reference: switch_gpu.cu:140-152
// (grid (n/16, n/16), block 16x16); grid-strided here so any grid works.
extern "C" __global__ void sgemm_naive(const float *__restrict__ A, const float *__restrict__ B,
                                       float *__restrict__ C, int M, int N, int K) {
    for (int row = blockIdx.y * blockDim.y + threadIdx.y; row < M; row += gridDim.y * blockDim.y)
        for (int col = blockIdx.x * blockDim.x + threadIdx.x; col < N; col += gridDim.x * blockDim.x) {
            float acc = 0.0f;
            for (int k = 0; k < K; k++) acc = __fadd_rn(acc, __fmul_rn(A[(size_t)row * K + k], B[(size_t)k * N + col]));
            C[(size_t)row * N + col] = acc;
        }
}

// Streaming read: out[i0] = sum over this thread's float4s of (x+y+z+w),
// `iters` passes.  Reference: switch_gpu.cu:41-54 (grid 512, block 256).
// Four independent 128-bit loads per thread are kept in flight.
extern "C" __global__ void membw_read4(const float4 *__restrict__ buf, float *__restrict__ out, int n4, int iters) {
    const long i0 = threadIdx.x + (long)blockIdx.x * blockDim.x;
    const long stride = (long)gridDim.x * blockDim.x;
    float acc = 0.f;
    for (int it = 0; it < iters; ++it) {
        long i = i0;
        for (; i + 3 * stride < n4; i += 4 * stride) {
            const float4 v0 = __ldcs(buf + i), v1 = __ldcs(buf + i + stride);
            const float4 v2 = __ldcs(buf + i + 2 * stride), v3 = __ldcs(buf + i + 3 * stride);
            acc += v0.x + v0.y + v0.z + v0.w;
            acc += v1.x + v1.y + v1.z + v1.w;
            acc += v2.x + v2.y + v2.z + v2.w;
            acc += v3.x + v3.y + v3.z + v3.w;
        }
        for (; i < n4; i += stride) {
            const float4 v = __ldcs(buf + i);
            acc += v.x + v.y + v.z + v.w;
        }
    }
    if (i0 < n4) out[i0] = acc;
}

// FP32 FMA throughput probe (the B200 counterpart of the reference's
// hand-PTX fma_bench, gpu_test.c:63-79): 8 independent FMA chains per
// thread, `iters` x 8 x 2 FLOP per thread.
extern "C" __global__ void fma_peak(float *__restrict__ out, int iters, float m, float c) {
    float a0 = threadIdx.x * 1e-3f, a1 = a0 + 1.f, a2 = a0 + 2.f, a3 = a0 + 3.f;
    float a4 = a0 + 4.f, a5 = a0 + 5.f, a6 = a0 + 6.f, a7 = a0 + 7.f;
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int u = 0; u < 16; u++) {
            a0 = fmaf(a0, m, c); a1 = fmaf(a1, m, c); a2 = fmaf(a2, m, c); a3 = fmaf(a3, m, c);
            a4 = fmaf(a4, m, c); a5 = fmaf(a5, m, c); a6 = fmaf(a6, m, c); a7 = fmaf(a7, m, c);
        }
    }
    out[blockIdx.x * blockDim.x + threadIdx.x] = a0 + a1 + a2 + a3 + a4 + a5 + a6 + a7;
}
