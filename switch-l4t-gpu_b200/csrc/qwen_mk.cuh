// qwen_mk.cuh -- the whole Qwen2.5-0.5B decode step as ONE persistent,
// cooperatively launched kernel (one CTA per SM).
//
// Why: a decode step is ~120 dependent matvec stages; as separate kernels
// each pays launch, ramp-up and a chain of dependent global round trips
// (measured ~6-13 us per kernel).  Here every stage is separated by a
// grid-wide barrier instead, and the weights -- which never depend on the
// activations -- are fetched ahead of the barriers:
//   * each warp copies its rows of the NEXT stage into its own shared-memory
//     region with cp.async right after finishing the current stage, i.e.
//     while it waits at the barrier, so after the barrier the weights are
//     already on chip;
//   * thread 0 of each CTA issues an L2 bulk prefetch of its whole slice of
//     the next layer (~200 KB per CTA, ~30 MB in total) so HBM streams
//     continuously underneath the barrier latency chain.
// Stages per layer (each CTA owns a contiguous block of rows of every matrix):
//   S1 RMSNorm(x) -> QKV rows (RoPE pairs) + bias + RoPE -> q, K/V cache
//   S2 attention partials: (head, T-split) items, split-local softmax
//   S3 combine partials -> att; O rows; x += O att
//   S4 RMSNorm(x) -> gate/up row pairs -> SwiGLU -> hid
//   S5 down rows (split-K over warps); x += down hid
// then final RMSNorm -> LM head rows (cp.async ring per warp) -> logits +
// argmax, and the step finalisation (next token, position).
//
// Barrier waits are bounded: after SB_MK_SPIN_LIMIT polls the kernel sets
// *err, drains its own copies and returns; the host reports the error.
#pragma once
#include "sb_attn.cuh"
#include "sb_finalize.cuh"
#include "sb_gemv.cuh"
#include "sb_mk_params.h"

namespace qmk {

constexpr int C = 896, NH = 14, NKV = 2, HD = 64, KVD = 128, QKV = 1152, FC = 4864, V = 151936, NL = 24;
constexpr int CTX_FILE = 8192;
constexpr int THREADS = 512, WARPS = 16;
constexpr long OFF_COS = (long)V * C * 2;
constexpr long OFF_SIN = OFF_COS + (long)CTX_FILE * (HD / 2) * 4;
constexpr long LBASE = OFF_SIN + (long)CTX_FILE * (HD / 2) * 4;
constexpr long LSTRIDE = (long)(C + QKV * C + QKV + C * C + C + 2 * FC * C + C * FC) * 2;
constexpr long OFF_LNF = LBASE + (long)NL * LSTRIDE;
// fp16-element offsets inside a layer
constexpr long L_INLN = 0, L_QKVW = C, L_QKVB = L_QKVW + (long)QKV * C, L_OW = L_QKVB + QKV;
constexpr long L_POST = L_OW + (long)C * C, L_GATEUP = L_POST + C, L_DOWN = L_GATEUP + (long)2 * FC * C;
constexpr int CPR = C / 8;            // 16-byte chunks per K=896 row (112)
constexpr int CPR_D = FC / 8;         // chunks per K=4864 row (608)
constexpr int WREG = 6 * C * 2;       // per-warp weight region: 6 rows of 896 fp16 (10752 B)
constexpr int LM_NB = 3;              // LM-head rows in flight per warp
constexpr long SPIN_LIMIT = 1L << 22; // barrier polls (~seconds) before giving up

// Typed view of SbMkParams.
struct Params {
    const unsigned short *w; // weight file image
    float *kv;               // [2][NL][ctx][KVD]
    float *x;                // residual [C]
    float *q;                // [C]
    float *part;             // attention partials [NH * splits][HD + 2]
    float *hid;              // [FC]
    float *logits;           // [V]
    SbStep *st;
    int *tokens;
    unsigned *bar;           // grid barrier counter, zero at launch
    int *err;                // set on a barrier timeout
    unsigned long long *trace;
    int ctx_cap;
    int with_logits;
    int splits;              // attention T-splits per head (<= gridDim.x / NH)
    int score_cap;           // positions per split the score buffer holds
    SB_DEV explicit Params(const SbMkParams &r)
        : w((const unsigned short *)r.w), kv((float *)r.kv), x((float *)r.x), q((float *)r.q),
          part((float *)r.part), hid((float *)r.hid), logits((float *)r.logits), st((SbStep *)r.st),
          tokens((int *)r.tokens), bar((unsigned *)r.bar), err((int *)r.err),
          trace((unsigned long long *)r.trace), ctx_cap(r.ctx_cap),
          with_logits(r.with_logits), splits(r.splits), score_cap(r.score_cap) {}
};

// ------------------------------------------------------------------ PTX helpers
SB_DEV unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
SB_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
SB_DEV void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
SB_DEV void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
SB_DEV void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
SB_DEV unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
SB_DEV unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Copy `nchunks` 16-byte chunks of one weight row (starting at chunk c0)
// into shared memory, warp-cooperatively.
SB_DEV void warp_copy_row(void *dst, const unsigned short *row, int c0, int nchunks) {
    const int lane = threadIdx.x & 31;
    const uint4 *src = reinterpret_cast<const uint4 *>(row) + c0;
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int c = lane; c < nchunks; c += 32) cp_async16(d + c, src + c);
}

// Grid-wide barrier: every CTA arrives once; returns false on timeout
// (after setting *err).  `target` = number of arrivals to wait for.
SB_DEV bool grid_sync(const Params &p, unsigned target, int *abort_s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long *tr = nullptr;
        if (p.trace) {
            const unsigned idx = target / gridDim.x;  // 1-based barrier number
            if (idx < 128) tr = p.trace + ((size_t)blockIdx.x * 128 + idx) * 2;
        }
        if (tr) tr[0] = globaltimer();
        __threadfence();
        atomicAdd(p.bar, 1u);
        long spins = 0;
        while (ld_acquire(p.bar) < target) {
            if (*(volatile int *)p.err) break;
            if (++spins > SPIN_LIMIT) { atomicExch(p.err, 1); break; }
        }
        *abort_s = *(volatile int *)p.err;
        if (tr) tr[1] = globaltimer();
    }
    __syncthreads();
    return *abort_s == 0;
}

// Contiguous share [lo, hi) of n units for CTA b of g.
SB_DEV void share(int n, int b, int g, int &lo, int &hi) {
    lo = (int)((long)n * b / g);
    hi = (int)((long)n * (b + 1) / g);
}

// dot of one smem row (K/8 chunks) with the split x planes, lane-strided,
// chunk range [c0, c1) of the plane index.
SB_DEV float smem_row_dot(const uint4 *row, const float4 *lo, const float4 *hi, int c0, int c1, int row_c0) {
    float acc = 0.0f;
    for (int c = c0 + (threadIdx.x & 31); c < c1; c += 32) acc = dot_chunk(WH(), row[c - row_c0], lo[c], hi[c], acc);
    return acc;
}

// Stage RMSNorm(x) * g into split planes (x read through L2: other CTAs wrote it).
SB_DEV void stage_rms(const float *x, const unsigned short *g, float4 *lo, float4 *hi, float *red, float eps) {
    float s = 0.0f;
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        const float v = __ldcg(x + i);
        s = fmaf(v, v, s);
    }
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(__fdiv_rn(s, (float)C) + eps);
    for (int c = threadIdx.x; c < CPR; c += blockDim.x) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = __fmul_rn(__fmul_rn(__ldcg(x + 8 * c + j), inv), h2f_ftz(g[8 * c + j]));
        lo[c] = make_float4(v[0], v[1], v[2], v[3]);
        hi[c] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// ------------------------------------------------------------------ the kernel
}  // namespace qmk

// grid: one CTA per SM (cooperative launch, >= 128 CTAs); block qmk::THREADS;
// dynamic smem qmk_smem_bytes(score_cap).
extern "C" __global__ void __launch_bounds__(qmk::THREADS, 1) qwen_decode_mk(const SbMkParams raw) {
    using namespace qmk;
    const Params p(raw);
    extern __shared__ __align__(16) unsigned char smem[];
    // layout: x planes (FC floats) | weight regions (WARPS * WREG) | scores | small
    float4 *xlo = reinterpret_cast<float4 *>(smem);
    float4 *xhi = xlo + CPR_D;                                    // planes sized for K = FC
    unsigned char *wbase = smem + (size_t)FC * 4;
    float *scores = reinterpret_cast<float *>(wbase + (size_t)WARPS * WREG);
    float *red = scores + p.score_cap;                            // 32 floats
    float *opart = red + 32;                                      // 8 x HD partial P.V
    float *ksum = opart + 8 * HD;                                 // WARPS floats for split-K reduce
    __shared__ int abort_s;
    __shared__ float m_s, l_s;
    __shared__ unsigned long long best_s;

    const int b = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char *wreg = wbase + (size_t)warp * WREG;
    const uint4 *wreg4 = reinterpret_cast<const uint4 *>(wreg);
    unsigned target = 0;
    if (threadIdx.x == 0) abort_s = 0;
    if (sb_step_idle(p.st)) return;  // uniform: every CTA reads the same state
    if (p.trace && threadIdx.x == 0) p.trace[(size_t)b * 256] = globaltimer();  // slot 0: start
    const int pos = p.st->pos, T = pos + 1;
    const int tok = p.tokens[pos];
    const float eps = 1e-6f;
    const unsigned short *emb = p.w;
    const float *cosT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_COS);
    const float *sinT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_SIN);

    // per-CTA shares (static over the step)
    int qp0, qp1, or0, or1, gp0, gp1;
    share(QKV / 2, b, G, qp0, qp1);  // RoPE pairs
    share(C, b, G, or0, or1);        // O rows and down rows
    share(FC, b, G, gp0, gp1);       // gate/up pairs

    auto layer_ptr = [&](int l) { return p.w + (LBASE / 2) + (long)l * (LSTRIDE / 2); };

    // L2 prefetch of this CTA's slices of layer l
    auto prefetch_layer = [&](int l) {
        if (threadIdx.x != 0 || l >= NL) return;
        const unsigned short *L = layer_ptr(l);
        for (int pp = qp0; pp < qp1; pp++) {  // QKV pair rows (few)
            const int h = pp / 32, i = pp % 32;
            l2_prefetch_bulk(L + L_QKVW + (long)(h * HD + i) * C, C * 2);
            l2_prefetch_bulk(L + L_QKVW + (long)(h * HD + 32 + i) * C, C * 2);
        }
        prefetch_rows(L + L_OW, C * 2, or0, or1, 1L << 20);
        prefetch_rows(L + L_GATEUP, C * 2, gp0, gp1, 1L << 20);
        prefetch_rows(L + L_GATEUP, C * 2, FC + gp0, FC + gp1, 1L << 20);
        prefetch_rows(L + L_DOWN, (long)FC * 2, or0, or1, 1L << 20);
    };

    // ---- stage weight copies (issued before the barrier that precedes use)
    auto copy_s1 = [&](int l) {  // warp w < npairs: pair qp0 + w, rows r, r+32
        const int pp = qp0 + warp;
        if (pp < qp1) {
            const int h = pp / 32, i = pp % 32;
            const unsigned short *W = layer_ptr(l) + L_QKVW;
            warp_copy_row(wreg, W + (long)(h * HD + i) * C, 0, CPR);
            warp_copy_row(wreg + C * 2, W + (long)(h * HD + 32 + i) * C, 0, CPR);
        }
        cp_commit();
    };
    auto copy_s3 = [&](int l) {  // O rows: warp w -> row or0 + w/2, half w%2
        const int r = or0 + warp / 2, half = warp % 2;
        if (r < or1) warp_copy_row(wreg, layer_ptr(l) + L_OW + (long)r * C, half * (CPR / 2), CPR / 2);
        cp_commit();
    };
    auto copy_s4 = [&](int l) {  // gate/up pairs gp0 + warp + 16k, k < 3
        const unsigned short *W = layer_ptr(l) + L_GATEUP;
        for (int k = 0; k < 3; k++) {
            const int i = gp0 + warp + WARPS * k;
            if (i < gp1) {
                warp_copy_row(wreg + (2 * k) * C * 2, W + (long)i * C, 0, CPR);
                warp_copy_row(wreg + (2 * k + 1) * C * 2, W + (long)(FC + i) * C, 0, CPR);
            }
        }
        cp_commit();
    };
    auto copy_s5 = [&](int l) {  // down rows: warp w -> row or0 + w/2, half w%2 of K
        const int r = or0 + warp / 2, half = warp % 2;
        if (r < or1) warp_copy_row(wreg, layer_ptr(l) + L_DOWN + (long)r * FC, half * (CPR_D / 2), CPR_D / 2);
        cp_commit();
    };

    // ---- prologue: x rows this CTA updates in S3 start as the embedding
    for (int r = or0 + threadIdx.x; r < or1; r += blockDim.x) p.x[r] = h2f_ftz(emb[(long)tok * C + r]);
    prefetch_layer(0);
    prefetch_layer(1);
    copy_s1(0);

    for (int l = 0; l < NL; l++) {
        const unsigned short *L = layer_ptr(l);
        float *kc = p.kv + (long)l * p.ctx_cap * KVD;
        float *vc = p.kv + (long)(NL + l) * p.ctx_cap * KVD;
        // ================= S1: RMSNorm -> QKV -> RoPE -> q / cache
        if (l > 0) {
            target += G;
            if (!grid_sync(p, target, &abort_s)) break;
        }
        prefetch_layer(l + 1);
        if (l == 0) {  // x = embedding row (nobody wrote the global x yet)
            float s = 0.0f;
            for (int i = threadIdx.x; i < C; i += blockDim.x) {
                const float v = h2f_ftz(emb[(long)tok * C + i]);
                s = fmaf(v, v, s);
            }
            s = block_sum(s, red);
            const float inv = 1.0f / sqrtf(__fdiv_rn(s, (float)C) + eps);
            for (int c = threadIdx.x; c < CPR; c += blockDim.x) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; j++)
                    v[j] = __fmul_rn(__fmul_rn(h2f_ftz(emb[(long)tok * C + 8 * c + j]), inv), h2f_ftz(L[L_INLN + 8 * c + j]));
                xlo[c] = make_float4(v[0], v[1], v[2], v[3]);
                xhi[c] = make_float4(v[4], v[5], v[6], v[7]);
            }
        } else {
            stage_rms(p.x, L + L_INLN, xlo, xhi, red, eps);
        }
        __syncthreads();
        cp_wait_all();
        __syncwarp();
        {
            const int pp = qp0 + warp;
            if (pp < qp1) {
                const int h = pp / 32, i = pp % 32;
                const int r0 = h * HD + i, r1 = r0 + 32;
                float a0 = warp_sum(smem_row_dot(wreg4, xlo, xhi, 0, CPR, 0));
                float a1 = warp_sum(smem_row_dot(wreg4 + CPR, xlo, xhi, 0, CPR, 0));
                if (lane == 0) {
                    float y0 = __fadd_rn(a0, h2f_ftz(L[L_QKVB + r0]));
                    float y1 = __fadd_rn(a1, h2f_ftz(L[L_QKVB + r1]));
                    if (h < NH + NKV) {
                        const float c = cosT[(long)pos * 32 + i], s = sinT[(long)pos * 32 + i];
                        const float o0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
                        const float o1 = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
                        y0 = o0;
                        y1 = o1;
                    }
                    if (h < NH) { p.q[r0] = y0; p.q[r1] = y1; }
                    else if (h < NH + NKV) { kc[(long)pos * KVD + r0 - C] = y0; kc[(long)pos * KVD + r1 - C] = y1; }
                    else { vc[(long)pos * KVD + r0 - C - KVD] = y0; vc[(long)pos * KVD + r1 - C - KVD] = y1; }
                }
            }
        }
        // ================= S2: attention partials
        target += G;
        if (!grid_sync(p, target, &abort_s)) break;
        copy_s3(l);  // O rows arrive while attention runs
        {
            const int S = p.splits;
            const int nsplit = min(S, (T + 7) / 8);
            const int slen = (T + nsplit - 1) / nsplit;
            for (int item = b; item < NH * nsplit; item += G) {
                const int h = item / nsplit, s = item % nsplit, g = h / (NH / NKV);
                const int t0 = s * slen, t1 = min(T, t0 + slen), n = max(0, t1 - t0);
                const float2 q2 = __ldcg(reinterpret_cast<const float2 *>(p.q + h * HD) + lane);
                for (int j = warp; j < n; j += WARPS) {
                    const float2 k2 = __ldcg(reinterpret_cast<const float2 *>(kc + (long)(t0 + j) * KVD + g * HD) + lane);
                    float d = fmaf(q2.x, k2.x, q2.y * k2.y);
                    d = warp_sum(d);
                    if (lane == 0) scores[j] = d * 0.125f;
                }
                __syncthreads();
                if (warp == 0) {
                    float m = -1e30f;
                    for (int j = lane; j < n; j += 32) m = fmaxf(m, scores[j]);
                    m = warp_max(m);
                    float sum = 0.0f;
                    for (int j = lane; j < n; j += 32) {
                        const float e = expf(scores[j] - m);
                        scores[j] = e;
                        sum += e;
                    }
                    sum = warp_sum(sum);
                    if (lane == 0) { m_s = m; l_s = sum; }
                }
                __syncthreads();
                {  // P.V: 8 position groups x 64 dims
                    const int d = threadIdx.x & 63, grp = threadIdx.x >> 6;
                    float acc = 0.0f;
                    for (int j = grp; j < n; j += 8) acc = fmaf(scores[j], __ldcg(vc + (long)(t0 + j) * KVD + g * HD + d), acc);
                    opart[grp * HD + d] = acc;
                }
                __syncthreads();
                if (threadIdx.x < HD) {
                    float o = 0.0f;
                    for (int k = 0; k < 8; k++) o += opart[k * HD + threadIdx.x];
                    float *pp = p.part + (long)(h * S + s) * (HD + 2);
                    pp[threadIdx.x] = o;
                    if (threadIdx.x == 0) { pp[HD] = m_s; pp[HD + 1] = l_s; }
                }
                __syncthreads();
            }
        }
        // ================= S3: combine -> att; O rows; x += O att
        target += G;
        if (!grid_sync(p, target, &abort_s)) break;
        {
            const int nsplit = min(p.splits, (T + 7) / 8);
            for (int o = threadIdx.x; o < C; o += blockDim.x) {
                const int h = o / HD, d = o % HD;
                const float *base = p.part + (long)(h * p.splits) * (HD + 2);
                float M = -1e30f;
                for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(base + (long)s * (HD + 2) + HD));
                float Lsum = 0.0f, acc = 0.0f;
                for (int s = 0; s < nsplit; s++) {
                    const float *pp = base + (long)s * (HD + 2);
                    const float w = expf(__ldcg(pp + HD) - M);
                    Lsum = fmaf(w, __ldcg(pp + HD + 1), Lsum);
                    acc = fmaf(w, __ldcg(pp + d), acc);
                }
                reinterpret_cast<float *>(o % 8 < 4 ? xlo : xhi)[(o / 8) * 4 + (o % 4)] = acc / Lsum;
            }
        }
        __syncthreads();
        cp_wait_all();
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a = 0.0f;
            if (r < or1) a = warp_sum(smem_row_dot(wreg4, xlo, xhi, half * (CPR / 2), (half + 1) * (CPR / 2), half * (CPR / 2)));
            if (lane == 0) ksum[warp] = a;
            __syncthreads();
            if (threadIdx.x < or1 - or0) {
                const int rr = or0 + threadIdx.x;
                const float y = ksum[2 * threadIdx.x] + ksum[2 * threadIdx.x + 1];
                p.x[rr] = __fadd_rn(__ldcg(p.x + rr), y);
            }
        }
        copy_s4(l);
        // ================= S4: RMSNorm -> gate/up -> SwiGLU -> hid
        target += G;
        if (!grid_sync(p, target, &abort_s)) break;
        stage_rms(p.x, L + L_POST, xlo, xhi, red, eps);
        __syncthreads();
        cp_wait_all();
        __syncwarp();
        for (int k = 0; k < 3; k++) {
            const int i = gp0 + warp + WARPS * k;
            if (i < gp1) {
                const float ag = warp_sum(smem_row_dot(wreg4 + (2 * k) * CPR, xlo, xhi, 0, CPR, 0));
                const float au = warp_sum(smem_row_dot(wreg4 + (2 * k + 1) * CPR, xlo, xhi, 0, CPR, 0));
                if (lane == 0) p.hid[i] = __fmul_rn(__fdiv_rn(ag, __fadd_rn(1.0f, expf(-ag))), au);
            }
        }
        copy_s5(l);
        // ================= S5: down rows (split-K over warp pairs); x += down hid
        target += G;
        if (!grid_sync(p, target, &abort_s)) break;
        for (int c = threadIdx.x; c < CPR_D; c += blockDim.x) {
            const float4 a = __ldcg(reinterpret_cast<const float4 *>(p.hid) + 2 * c);
            const float4 bb = __ldcg(reinterpret_cast<const float4 *>(p.hid) + 2 * c + 1);
            xlo[c] = a;
            xhi[c] = bb;
        }
        __syncthreads();
        cp_wait_all();
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a = 0.0f;
            if (r < or1)
                a = warp_sum(smem_row_dot(wreg4, xlo, xhi, half * (CPR_D / 2), (half + 1) * (CPR_D / 2), half * (CPR_D / 2)));
            if (lane == 0) ksum[warp] = a;
            __syncthreads();
            if (threadIdx.x < or1 - or0) {
                const int rr = or0 + threadIdx.x;
                const float y = ksum[2 * threadIdx.x] + ksum[2 * threadIdx.x + 1];
                p.x[rr] = __fadd_rn(__ldcg(p.x + rr), y);
            }
        }
        if (l + 1 < NL) copy_s1(l + 1);
    }
    if (abort_s) {
        cp_wait_all();
        return;
    }
    // ================= LM head + argmax
    target += G;
    if (!grid_sync(p, target, &abort_s)) { cp_wait_all(); return; }
    if (p.with_logits) {
        stage_rms(p.x, p.w + OFF_LNF / 2, xlo, xhi, red, eps);
        if (threadIdx.x == 0) best_s = 0ull;
        __syncthreads();
        int v0, v1;
        share(V, b, G, v0, v1);
        // per warp: rows v0 + warp + 16k through a ring of LM_NB row buffers
        unsigned long long best = 0ull;
        int issued = 0;
        for (int k = 0; k < LM_NB; k++) {
            const int r = v0 + warp + WARPS * k;
            if (r < v1) warp_copy_row(wreg + k * C * 2, emb + (long)r * C, 0, CPR);
            cp_commit();
            issued++;
        }
        for (int k = 0;; k++) {
            const int r = v0 + warp + WARPS * k;
            if (r >= v1) break;
            cp_wait<LM_NB - 1>();
            __syncwarp();
            const int slot = k % LM_NB;
            const float a = warp_sum(smem_row_dot(wreg4 + slot * CPR, xlo, xhi, 0, CPR, 0));
            if (lane == 0) p.logits[r] = a;
            const unsigned long long key = argmax_key(a, r);
            best = key > best ? key : best;
            __syncwarp();
            const int rn = v0 + warp + WARPS * (k + LM_NB);
            if (rn < v1) warp_copy_row(wreg + slot * C * 2, emb + (long)rn * C, 0, CPR);
            cp_commit();
        }
        cp_wait_all();
        if (lane == 0 && best) atomicMax(&best_s, best);
        __syncthreads();
        if (threadIdx.x == 0 && best_s) atomicMax(&p.st->key, best_s);
        target += G;
        if (!grid_sync(p, target, &abort_s)) return;
    }
    // ================= finalize (one thread of CTA 0), as sb_finalize
    if (b == 0 && threadIdx.x == 0) {
        SbStep *st = p.st;
        const int pp = st->pos;
        if (p.with_logits) {
            const int nxt = argmax_key_index(st->key);
            st->key = 0ull;
            if (pp + 1 >= st->n_prompt && pp + 1 < st->n_end) {
                p.tokens[pp + 1] = nxt;
                st->n_generated += 1;
                if (st->stop_on_eos && (nxt == st->eos0 || nxt == st->eos1)) st->done = 1;
            }
        }
        st->pos = pp + 1;
        if (st->pos >= st->n_end - 1) st->done = 1;
    }
}
