// gpt2_mk.cuh -- the whole GPT-2 (124M) decode step as ONE persistent,
// cooperatively launched kernel (one CTA per SM): the GPT-2 counterpart of
// qwen_decode_mk, with the same stage hand-off through flagged words
// (sb_mk_common.cuh) and the same weight staging (each warp copies its rows
// of the next stage into shared memory with TMA bulk copies as soon as its
// current rows are consumed; one lane issues L2 prefetches of the next
// layer).  The arithmetic is the reference's cpu_forward
// (gpu-llm/engine/gpt2_engine.c:363-421): FP32 weights, LayerNorm with the
// mean and then the centred variance, biases on every product, tanh-GELU,
// 12-head attention, learned position embeddings, tied LM head.
//
// Stages per layer (each CTA owns a contiguous block of rows of every matrix):
//   S1 LayerNorm(x) -> QKV rows + bias -> q, k, v words (k, v into the cache)
//   S2 attention partials: (head, T-split) items, one per CTA
//   S3 combine partials -> att; O rows + bias; x += -> x words (own rows)
//   S4 LayerNorm(x) -> fc rows + bias -> GELU -> hid words
//   S5 proj rows (split-K over warp pairs) + bias; x += -> x words
// then final LayerNorm -> LM head rows -> logits + argmax; CTA 0 finalises.
// Waits are bounded (LL_SPIN_LIMIT polls); on a timeout *err is set, the
// CTA drains its bulk copies and returns.
#pragma once
#include "sb_finalize.cuh"
#include "sb_gemv.cuh"
#include "sb_mk_common.cuh"

namespace g2mk {
using namespace mkc;

constexpr int C = 768, NH = 12, HD = 64, QKV = 3 * C, FC = 3072, V = 50257, NL = 12, CTX_FILE = 1024;
constexpr int THREADS = 512, WARPS = 16;
// float offsets in the weight file (gpt2_engine.c:50-70)
constexpr long OFF_WPE = (long)V * C;
constexpr long LBASE = OFF_WPE + (long)CTX_FILE * C;
constexpr long LAYER = 2L * C + 3L * C * C + 3L * C + (long)C * C + C + 2L * C + (long)FC * C + FC + (long)FC * C + C;
constexpr long OFF_LNFW = LBASE + (long)NL * LAYER, OFF_LNFB = OFF_LNFW + C;
constexpr long L_LN1W = 0, L_LN1B = C, L_QKVW = 2L * C, L_QKVB = L_QKVW + 3L * C * C, L_AOW = L_QKVB + 3L * C;
constexpr long L_AOB = L_AOW + (long)C * C, L_LN2W = L_AOB + C, L_LN2B = L_LN2W + C, L_FCW = L_LN2B + C;
constexpr long L_FCB = L_FCW + (long)FC * C, L_PROJW = L_FCB + FC, L_PROJB = L_PROJW + (long)FC * C;
constexpr int CR = C / 4;             // float4 chunks per K=768 row (192)
constexpr int CR_F = FC / 4;          // chunks per K=3072 row (768)
constexpr int ROWB = C * 4;           // bytes of one K=768 row (3072)
constexpr int WHEAD = 3 * ROWB;       // per-warp slot: 3 rows (QKV, fc, proj half, LM ring)
constexpr int WREG = WHEAD + ROWB / 2;// + the O half-row: 10752 B per warp
constexpr int LM_NB = 3;
constexpr int SPLITS_MAX = SB_MK_SPLITS_MAX;
constexpr int PW = HD + 2;
constexpr int LL_X = 0, LL_QKV = LL_X + C, LL_HID = LL_QKV + QKV, LL_PART = LL_HID + FC;
static_assert(LL_PART + NH * SPLITS_MAX * PW <= SB_MK_LL_WORDS, "flagged-word area");
static_assert(LL_QKV % 2 == 0 && LL_HID % 2 == 0 && LL_PART % 2 == 0, "pairs stay 16-byte aligned");
constexpr int HID_PAIRS = (FC / 2 + THREADS - 1) / THREADS;  // 3
static_assert(C >= THREADS && NH * SPLITS_MAX <= THREADS,
              "the combine polls each (m, l) pair with the o words of dim tid");

// R fp32 rows at base + r*stride (float4 units) against x (float4 chunks),
// chunk range [c0, c1), row data starting at chunk row_c0; per-lane partials.
template <int R>
SB_DEV void rows_dot_f32(const float4 *base, int stride, int nvalid, const float4 *xs, int c0, int c1, int row_c0,
                         float (&out)[R]) {
    unsigned long long acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0ull;
    for (int c = c0 + (threadIdx.x & 31); c < c1; c += 32) {
        const float4 x = xs[c];
#pragma unroll
        for (int r = 0; r < R; r++)
            if (r < nvalid) {
                const float4 w = base[r * stride + c - row_c0];
                acc[r] = ffma2(f2_pack(w.x, w.y), f2_pack(x.x, x.y), acc[r]);
                acc[r] = ffma2(f2_pack(w.z, w.w), f2_pack(x.z, x.w), acc[r]);
            }
    }
#pragma unroll
    for (int r = 0; r < R; r++) out[r] = f2_sum(acc[r]);
}

// LayerNorm from registers (thread t < C/2 holds elements 2t, 2t+1 in xv):
// mean, then the centred variance (the reference's order of operations),
// y = ((x - mean) * inv) * w + b written to xs (plain float layout).
SB_DEV void ln_regs(float2 xv, const float *w, const float *bias, float *xs, float *red, float eps) {
    const int t = threadIdx.x;
    const bool act = t < C / 2;
    const float mean = __fdiv_rn(block_sum1(act ? xv.x + xv.y : 0.f, red, 0), (float)C);
    const float d0 = xv.x - mean, d1 = xv.y - mean;
    const float var = __fdiv_rn(block_sum1(act ? fmaf(d0, d0, d1 * d1) : 0.f, red, 16), (float)C);
    const float inv = 1.0f / sqrtf(var + eps);
    if (act) {
        const float2 g = *reinterpret_cast<const float2 *>(w + 2 * t), bb = *reinterpret_cast<const float2 *>(bias + 2 * t);
        *reinterpret_cast<float2 *>(xs + 2 * t) =
            make_float2(__fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv.x, mean), inv), g.x), bb.x),
                        __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv.y, mean), inv), g.y), bb.y));
    }
}

// tanh-GELU, every product and sum rounded in the reference C's order
// (gpt2_engine.c:406-410).
SB_DEV float gelu_r(float v) {
    const float p = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    const float t = __fmul_rn(0.7978845608f, __fadd_rn(v, p));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(t)));
}

}  // namespace g2mk

// grid: one CTA per SM (cooperative launch, >= 128 CTAs); block g2mk::THREADS;
// dynamic smem: FC*4 + WARPS*WREG + round4(score_cap)*4
//               + (32 + WARPS*64 + WARPS + NH*SPLITS_MAX*2)*4 bytes.
extern "C" __global__ void __launch_bounds__(g2mk::THREADS, 1) gpt2_decode_mk(const SbMkParams raw) {
    using namespace g2mk;
    const Params p(raw);
    extern __shared__ __align__(16) unsigned char smem[];
    float *xs = reinterpret_cast<float *>(smem);  // activations for K up to FC
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    unsigned char *wbase = smem + (size_t)FC * 4;
    float *scores = reinterpret_cast<float *>(wbase + (size_t)WARPS * WREG);
    float *red = scores + ((p.score_cap + 3) & ~3);
    float *opart = red + 32;
    float *ksum = opart + WARPS * HD;
    float *mlv = ksum + WARPS;
    __shared__ float wmax_s[WARPS], xown[8], rbias[8];
    __shared__ unsigned long long best_s;
    __shared__ __align__(8) uint64_t mbar[WARPS][2 + LM_NB];

    const int b = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    unsigned char *wreg = wbase + (size_t)warp * WREG;
    const float4 *wreg4 = reinterpret_cast<const float4 *>(wreg);
    if (sb_step_idle(p.st)) return;
    if (lane == 0)
        for (int i = 0; i < 2 + LM_NB; i++) mbar_init(&mbar[warp][i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    if (p.trace && tid == 0) p.trace[(size_t)b * 256] = globaltimer();
    const unsigned seq = p.sync[0];
    auto epoch = [&](int l, int s) { return (seq << 7) | (unsigned)(l * 5 + s + 1); };
    auto stamp = [&](int l, int s, int which) {
        if (p.trace && tid == 0) p.trace[(size_t)b * 256 + 1 + 2 * (l * 5 + s) + which] = globaltimer();
    };
    const int pos = p.st->pos, T = pos + 1;
    const int tok = p.tokens[pos];
    const float eps = 1e-5f;
    const float *W = reinterpret_cast<const float *>(p.w);
    const float *wte = W, *wpe = W + OFF_WPE;
    const bool xact = tid < C / 2;
    u64 *const llx = p.ll + LL_X, *const llqkv = p.ll + LL_QKV, *const llhid = p.ll + LL_HID;
    u64 *const llpart = p.ll + LL_PART;

    int q0, q1, or0, or1, f0, f1;
    share(QKV, b, G, q0, q1);  // QKV rows (<= 2 per warp)
    share(C, b, G, or0, or1);  // O and proj rows: this CTA's residual rows
    share(FC, b, G, f0, f1);   // fc rows (<= 2 per warp)
    const int nsplit = max(1, min(min(p.splits, SPLITS_MAX), (T + 47) / 48));
    const int slen = (T + nsplit - 1) / nsplit;
    auto layer_ptr = [&](int l) { return W + LBASE + (long)l * LAYER; };

    auto prefetch_piece = [&](int l, int piece) {
        if (l >= NL) return;
        const float *L = layer_ptr(l);
        const int fmid = f0 + (f1 - f0) / 2, dmid = or0 + (or1 - or0) / 2;
        switch (piece) {
        case 0:
            prefetch_rows(L + L_QKVW, ROWB, q0, q1, 1L << 20);
            prefetch_rows(L + L_AOW, ROWB, or0, or1, 1L << 20);
            break;
        case 1: prefetch_rows(L + L_FCW, ROWB, f0, fmid, 1L << 20); break;
        case 2: prefetch_rows(L + L_FCW, ROWB, fmid, f1, 1L << 20); break;
        case 3: prefetch_rows(L + L_PROJW, (long)FC * 4, or0, dmid, 1L << 20); break;
        default: prefetch_rows(L + L_PROJW, (long)FC * 4, dmid, or1, 1L << 20); break;
        }
    };
    const bool prefetcher = (warp == WARPS - 2 && lane == 0);

    unsigned phase = 0, pend = 0;
    uint64_t *mb = mbar[warp];
    auto fence_async = [&]() {
        if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    };
    auto issue_begin = [&](int i, unsigned bytes) {
        mbar_expect_tx(&mb[i], bytes);
        pend |= 1u << i;
    };
    auto wait_slot = [&](int i) {
        if (!mbar_wait(&mb[i], (phase >> i) & 1u) && lane == 0) atomicExch(p.err, 2);
        phase ^= 1u << i;
        pend &= ~(1u << i);
    };
    const int nq = max(0, (q1 - q0 - warp + WARPS - 1) / WARPS);  // this warp's QKV rows (<= 2)
    const int nf = max(0, (f1 - f0 - warp + WARPS - 1) / WARPS);  // this warp's fc rows (<= 2)
    auto copy_s1 = [&](int l) {  // QKV rows q0 + warp + 16k
        if (lane != 0) return;
        issue_begin(0, (unsigned)nq * ROWB);
        for (int k = 0; k < nq; k++) bulk_g2s(wreg + k * ROWB, layer_ptr(l) + L_QKVW + (long)(q0 + warp + WARPS * k) * C, ROWB, &mb[0]);
    };
    auto copy_s3 = [&](int l) {  // O half-row: row or0 + w/2, half w%2 (tail slot)
        if (lane != 0) return;
        const int r = or0 + warp / 2, half = warp % 2;
        issue_begin(1, r < or1 ? ROWB / 2 : 0);
        if (r < or1) bulk_g2s(wreg + WHEAD, layer_ptr(l) + L_AOW + (long)r * C + half * (C / 2), ROWB / 2, &mb[1]);
    };
    auto copy_s4_piece = [&](int l, int k) {  // fc rows f0 + warp + 16k; byte count announced with k = 0
        if (lane != 0) return;
        if (k == 0) issue_begin(0, (unsigned)nf * ROWB);
        if (k < nf) bulk_g2s(wreg + k * ROWB, layer_ptr(l) + L_FCW + (long)(f0 + warp + WARPS * k) * C, ROWB, &mb[0]);
    };
    auto copy_s5 = [&](int l) {  // proj half-row: row or0 + w/2, half w%2 of K = 3072
        if (lane != 0) return;
        const int r = or0 + warp / 2, half = warp % 2;
        issue_begin(0, r < or1 ? FC * 2 : 0);
        if (r < or1) bulk_g2s(wreg, layer_ptr(l) + L_PROJW + (long)r * FC + half * (FC / 2), FC * 2, &mb[0]);
    };
    // split-K (2 warps per row) sum + bias (rbias, loaded ahead) + residual,
    // published as x words of epoch e
    auto resid_update = [&](float a, unsigned e) {
        if (lane == 0) ksum[warp] = a;
        __syncthreads();
        if (tid < or1 - or0) {
            const float y = __fadd_rn(ksum[2 * tid] + ksum[2 * tid + 1], rbias[tid]);
            const float xn = __fadd_rn(xown[tid], y);
            xown[tid] = xn;
            // test hook: the stalled CTA withholds its layer-0 outputs
            if (!(p.test_stall == b + 1 && e == epoch(0, 4))) ll_put(llx + or0 + tid, xn, e);
        }
    };
    float2 xv = make_float2(0.f, 0.f);
    auto wait_x = [&](unsigned e) {
        bool ok = true;
        if (xact) ok = ll_wait2(llx + 2 * tid, e, xv.x, xv.y, p.err);
        return !__syncthreads_or(!ok);
    };
    bool aborted = false;

    // ---- prologue: x = wte[token] + wpe[pos]
    if (tid < or1 - or0) xown[tid] = __fadd_rn(wte[(long)tok * C + or0 + tid], wpe[(long)pos * C + or0 + tid]);
    if (xact) {
        const float2 a = *reinterpret_cast<const float2 *>(wte + (long)tok * C + 2 * tid);
        const float2 c2 = *reinterpret_cast<const float2 *>(wpe + (long)pos * C + 2 * tid);
        xv = make_float2(__fadd_rn(a.x, c2.x), __fadd_rn(a.y, c2.y));
    }
    if (prefetcher)
        for (int piece = 0; piece < 5; piece++) prefetch_piece(0, piece);
    fence_async();
    copy_s1(0);
    float qb[2] = {0.f, 0.f};  // this warp's QKV row biases (lane 0)
    auto s1_consts = [&](int l) {
        if (lane == 0)
            for (int k = 0; k < nq; k++) qb[k] = layer_ptr(l)[L_QKVB + q0 + warp + WARPS * k];
    };
    s1_consts(0);

    for (int l = 0; l < NL; l++) {
        const float *L = layer_ptr(l);
        float *kc = p.kv + (long)l * p.ctx_cap * C;
        float *vc = p.kv + (long)(NL + l) * p.ctx_cap * C;
        // ================= S1: LayerNorm -> QKV + bias -> q, k, v words
        if (l > 0 && !wait_x(epoch(l - 1, 4))) { aborted = true; break; }
        stamp(l, 0, 0);
        ln_regs(xv, L + L_LN1W, L + L_LN1B, xs, red, eps);
        __syncthreads();
        // (An L2 prefetch of the LM-head rows during the last layers measured
        // 5 us per token slower: it competes with those layers' weights.)
        if (prefetcher) prefetch_piece(l + 1, 0);
        wait_slot(0);
        __syncwarp();
        {
            float a[2];
            rows_dot_f32<2>(wreg4, CR, nq, xs4, 0, CR, 0, a);
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const float d = warp_sum(a[k]);
                if (k < nq && lane == 0) {
                    const int r = q0 + warp + WARPS * k;
                    const float y = __fadd_rn(d, qb[k]);
                    ll_put(llqkv + r, y, epoch(l, 0));
                    if (r >= 2 * C) vc[(long)pos * C + r - 2 * C] = y;
                    else if (r >= C) kc[(long)pos * C + r - C] = y;
                }
            }
        }
        stamp(l, 0, 1);
        const bool has_item = b < NH * nsplit;
        auto issue_s3_s4 = [&]() {
            fence_async();
            copy_s3(l);
            copy_s4_piece(l, 0);
            if (prefetcher) prefetch_piece(l + 1, 1);
        };
        if (!has_item) issue_s3_s4();
        // ================= S2: attention partials (12 heads, MHA)
        const unsigned e_qkv = epoch(l, 0);
        for (int item = b; item < NH * nsplit; item += G) {
            const int h = item / nsplit, s = item % nsplit;
            const int t0 = s * slen, t1 = min(T, t0 + slen), n = max(0, t1 - t0);
            const u64 *kcur = llqkv + C + h * HD + 2 * lane, *vcur = llqkv + 2 * C + h * HD + 2 * lane;
            __syncthreads();
            float2 kk[4], vv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int t = t0 + warp + WARPS * k;
                kk[k] = vv[k] = make_float2(0.f, 0.f);
                if (t < t1 && t < pos) {
                    kk[k] = __ldcg(reinterpret_cast<const float2 *>(kc + (long)t * C + h * HD) + lane);
                    vv[k] = __ldcg(reinterpret_cast<const float2 *>(vc + (long)t * C + h * HD) + lane);
                }
            }
            float2 *qkv_s = reinterpret_cast<float2 *>(xs);  // free until S3 writes the attention output
            bool ok = true;
            if (warp == 0) {  // q (and the current k, v) requested together: one round trip
                const bool cur = t1 == T;
                const u64 *qw = llqkv + h * HD + 2 * lane;
                for (long spin = 0;; spin++) {
                    u64 w[6];
                    ll_get2(qw, w[0], w[1]);
                    if (cur) {
                        ll_get2(kcur, w[2], w[3]);
                        ll_get2(vcur, w[4], w[5]);
                    }
                    bool all = ll_is(w[0], e_qkv) && ll_is(w[1], e_qkv);
                    if (cur) all = all && ll_is(w[2], e_qkv) && ll_is(w[3], e_qkv) && ll_is(w[4], e_qkv) && ll_is(w[5], e_qkv);
                    if (all) {
                        qkv_s[lane] = make_float2(ll_val(w[0]), ll_val(w[1]));
                        if (cur) {
                            qkv_s[32 + lane] = make_float2(ll_val(w[2]), ll_val(w[3]));
                            qkv_s[64 + lane] = make_float2(ll_val(w[4]), ll_val(w[5]));
                        }
                        break;
                    }
                    if (!ll_keep_polling(spin, p.err)) { ok = false; break; }
                }
            }
            if (__syncthreads_or(!ok)) { aborted = true; break; }
            const float2 q2 = qkv_s[lane];
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (t0 + warp + WARPS * k == pos) {
                    kk[k] = qkv_s[32 + lane];
                    vv[k] = qkv_s[64 + lane];
                }
            float sc[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                sc[k] = -1e30f;
                if (warp + WARPS * k < n) sc[k] = warp_sum(fmaf(q2.x, kk[k].x, q2.y * kk[k].y)) * 0.125f;
            }
            float2 vpos = make_float2(0.f, 0.f);
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) {
                const int t = t0 + j;
                float2 k2;
                if (t == pos) {
                    k2 = qkv_s[32 + lane];
                    vpos = qkv_s[64 + lane];
                } else {
                    k2 = __ldcg(reinterpret_cast<const float2 *>(kc + (long)t * C + h * HD) + lane);
                }
                const float d = warp_sum(fmaf(q2.x, k2.x, q2.y * k2.y)) * 0.125f;
                if (lane == 0) scores[j] = d;
            }
            // each warp keeps its own softmax (max, sum, P.V); the CTA combines
            // the sixteen once
            float wm = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
            __syncwarp();
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) wm = fmaxf(wm, scores[j]);
            float lsum = 0.f;
            float2 o = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (warp + WARPS * k < n) {
                    const float e = expf(sc[k] - wm);
                    lsum += e;
                    o.x = fmaf(e, vv[k].x, o.x);
                    o.y = fmaf(e, vv[k].y, o.y);
                }
            }
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) {
                const int t = t0 + j;
                const float e = expf(scores[j] - wm);
                lsum += e;
                const float2 v2 = t == pos ? vpos : __ldcg(reinterpret_cast<const float2 *>(vc + (long)t * C + h * HD) + lane);
                o.x = fmaf(e, v2.x, o.x);
                o.y = fmaf(e, v2.y, o.y);
            }
            reinterpret_cast<float2 *>(opart + warp * HD)[lane] = o;
            if (lane == 0) {
                ksum[warp] = lsum;
                wmax_s[warp] = wm;
            }
            __syncthreads();
            if (tid < HD) {
                float M = -1e30f;
#pragma unroll
                for (int w = 0; w < WARPS; w++) M = fmaxf(M, wmax_s[w]);
                float acc = 0.f, ls = 0.f;
#pragma unroll
                for (int w = 0; w < WARPS; w++) {
                    const float f = expf(wmax_s[w] - M);
                    acc = fmaf(f, opart[w * HD + tid], acc);
                    ls = fmaf(f, ksum[w], ls);
                }
                u64 *pw = llpart + (long)(h * SPLITS_MAX + s) * PW;
                const unsigned e = epoch(l, 1);
                ll_put(pw + tid, acc, e);
                if (tid == 0) {
                    ll_put(pw + HD, M, e);
                    ll_put(pw + HD + 1, ls, e);
                }
            }
            // (the next item's first barrier, or S3's poll barrier, orders
            // the combine's reads before opart / ksum are rewritten)
        }
        if (aborted) break;
        stamp(l, 1, 1);
        if (has_item) issue_s3_s4();
        // ================= S3: combine partials -> att; O rows + bias; x +=
        if (tid < or1 - or0) rbias[tid] = L[L_AOB + or0 + tid];
        copy_s4_piece(l, 1);
        if (prefetcher) prefetch_piece(l + 1, 2);
        {
            const unsigned e = epoch(l, 1);
            bool ok = true;
            // this thread's (m, l) pair (item tid < NH*nsplit <= THREADS) is
            // polled together with its o words below
            const u64 *mlw = llpart + (long)((tid / nsplit) * SPLITS_MAX + tid % nsplit) * PW + HD;
            bool ml_done = tid >= NH * nsplit;
            float ov[2][SPLITS_MAX];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int d = tid + THREADS * u;
                if (d >= C) break;
                const u64 *base = llpart + (long)((d / HD) * SPLITS_MAX) * PW + (d % HD);
                for (long spin = 0; ok; spin++) {
                    bool all = true;
                    u64 m0 = 0ull, m1 = 0ull;
                    if (!ml_done) ll_get2(mlw, m0, m1);
#pragma unroll
                    for (int s = 0; s < SPLITS_MAX; s++) {
                        ov[u][s] = 0.f;
                        if (s < nsplit) {
                            const u64 wv = ll_get(base + (long)s * PW);
                            all = all && ll_is(wv, e);
                            ov[u][s] = ll_val(wv);
                        }
                    }
                    if (!ml_done) {
                        if (ll_is(m0, e) && ll_is(m1, e)) {
                            mlv[2 * tid] = ll_val(m0);
                            mlv[2 * tid + 1] = ll_val(m1);
                            ml_done = true;
                        } else {
                            all = false;
                        }
                    }
                    if (all) break;
                    ok = ll_keep_polling(spin, p.err);
                }
            }
            if (__syncthreads_or(!ok)) { aborted = true; break; }
            stamp(l, 2, 0);
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int d = tid + THREADS * u;
                if (d >= C) break;
                const int h = d / HD;
                float M = -1e30f;
                for (int s = 0; s < nsplit; s++) M = fmaxf(M, mlv[2 * (h * nsplit + s)]);
                float acc = 0.f, Lsum = 0.f;
#pragma unroll
                for (int s = 0; s < SPLITS_MAX; s++) {
                    if (s < nsplit) {
                        const float wgt = expf(mlv[2 * (h * nsplit + s)] - M);
                        Lsum = fmaf(wgt, mlv[2 * (h * nsplit + s) + 1], Lsum);
                        acc = fmaf(wgt, ov[u][s], acc);
                    }
                }
                xs[d] = acc / Lsum;
            }
        }
        __syncthreads();
        wait_slot(1);
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            rows_dot_f32<1>(reinterpret_cast<const float4 *>(wreg + WHEAD), 0, r < or1 ? 1 : 0, xs4, half * (CR / 2),
                            (half + 1) * (CR / 2), half * (CR / 2), a);
            resid_update(warp_sum(a[0]), epoch(l, 2));
        }
        stamp(l, 2, 1);
        // ================= S4: LayerNorm -> fc + bias -> GELU -> hid words
        float fb[2] = {0.f, 0.f};
        if (lane == 0)
            for (int k = 0; k < nf; k++) fb[k] = L[L_FCB + f0 + warp + WARPS * k];
        if (prefetcher) prefetch_piece(l + 1, 3);
        if (!wait_x(epoch(l, 2))) { aborted = true; break; }
        stamp(l, 3, 0);
        ln_regs(xv, L + L_LN2W, L + L_LN2B, xs, red, eps);
        __syncthreads();
        wait_slot(0);
        __syncwarp();
        {
            float a[2];
            rows_dot_f32<2>(wreg4, CR, nf, xs4, 0, CR, 0, a);
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const float d = warp_sum(a[k]);
                if (k < nf && lane == 0) ll_put(llhid + f0 + warp + WARPS * k, gelu_r(__fadd_rn(d, fb[k])), epoch(l, 3));
            }
        }
        stamp(l, 3, 1);
        fence_async();
        copy_s5(l);
        // ================= S5: proj rows (split-K over warp pairs) + bias; x +=
        if (tid < or1 - or0) rbias[tid] = L[L_PROJB + or0 + tid];
        if (prefetcher) prefetch_piece(l + 1, 4);
        {
            const unsigned e = epoch(l, 3);
            float2 hv[HID_PAIRS];
            bool ok = true;
            for (long spin = 0; ok; spin++) {
                bool all = true;
#pragma unroll
                for (int k = 0; k < HID_PAIRS; k++) {
                    const int u = tid + THREADS * k;
                    if (u < FC / 2) {
                        u64 w0, w1;
                        ll_get2(llhid + 2 * u, w0, w1);
                        all = all && ll_is(w0, e) && ll_is(w1, e);
                        hv[k] = make_float2(ll_val(w0), ll_val(w1));
                    }
                }
                if (all) break;
                ok = ll_keep_polling(spin, p.err);
            }
#pragma unroll
            for (int k = 0; k < HID_PAIRS; k++) {
                const int u = tid + THREADS * k;
                if (u < FC / 2) *reinterpret_cast<float2 *>(xs + 2 * u) = hv[k];
            }
            if (__syncthreads_or(!ok)) { aborted = true; break; }
        }
        stamp(l, 4, 0);
        wait_slot(0);
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            rows_dot_f32<1>(wreg4, 0, r < or1 ? 1 : 0, xs4, half * (CR_F / 2), (half + 1) * (CR_F / 2), half * (CR_F / 2), a);
            resid_update(warp_sum(a[0]), epoch(l, 4));
        }
        stamp(l, 4, 1);
        if (l + 1 < NL) {
            fence_async();
            copy_s1(l + 1);
            s1_consts(l + 1);
        }
    }
    if (aborted) {
        if (lane == 0)
            for (int i = 0; i < 2 + LM_NB; i++)
                if ((pend >> i) & 1u) mbar_wait(&mb[i], (phase >> i) & 1u);
        return;
    }
    // ================= final LayerNorm -> LM head (tied wte) + argmax
    if (p.with_logits) {
        if (tid == 0) best_s = 0ull;
        if (!wait_x(epoch(NL - 1, 4))) {
            if (lane == 0)
                for (int i = 0; i < 2 + LM_NB; i++)
                    if ((pend >> i) & 1u) mbar_wait(&mb[i], (phase >> i) & 1u);
            return;
        }
        ln_regs(xv, W + OFF_LNFW, W + OFF_LNFB, xs, red, eps);
        __syncthreads();
        int v0, v1;
        share(V, b, G, v0, v1);
        unsigned long long best = 0ull;
        fence_async();
        for (int k = 0; k < LM_NB; k++) {
            const int r = v0 + warp + WARPS * k;
            if (r < v1 && lane == 0) {
                issue_begin(2 + k, ROWB);
                bulk_g2s(wreg + k * ROWB, wte + (long)r * C, ROWB, &mb[2 + k]);
            }
        }
        for (int k = 0;; k++) {
            const int r = v0 + warp + WARPS * k;
            if (r >= v1) break;
            const int slot = k % LM_NB;
            wait_slot(2 + slot);
            __syncwarp();
            float a[1];
            rows_dot_f32<1>(reinterpret_cast<const float4 *>(wreg + slot * ROWB), 0, 1, xs4, 0, CR, 0, a);
            const float dotv = warp_sum(a[0]);
            if (lane == 0) p.logits[r] = dotv;
            const unsigned long long key = argmax_key(dotv, r);
            best = key > best ? key : best;
            __syncwarp();
            const int rn = v0 + warp + WARPS * (k + LM_NB);
            if (rn < v1 && lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_begin(2 + slot, ROWB);
                bulk_g2s(wreg + slot * ROWB, wte + (long)rn * C, ROWB, &mb[2 + slot]);
            }
        }
        if (lane == 0 && best) atomicMax(&best_s, best);
        __syncthreads();
        if (tid == 0) {
            if (best_s) atomicMax(&p.st->key, best_s);
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.sync + 1) : "memory");
        }
        if (b != 0 || tid != 0) return;
        for (long spin = 0; ld_acquire(p.sync + 1) < (unsigned)G; spin++)
            if (!ll_keep_polling(spin, p.err)) return;
        p.sync[1] = 0u;
    } else if (b != 0 || tid != 0) {
        return;
    }
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
    p.sync[0] = seq + 1u;
}
