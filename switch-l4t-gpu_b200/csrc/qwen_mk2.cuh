// qwen_mk2.cuh -- the Qwen2.5-0.5B decode step as one persistent kernel,
// with the MLP down projection split along its inner dimension.
//
// The stages, the flagged-word hand-off, the weight staging and the bounded
// waits are those of qwen_decode_mk (qwen_mk.cuh).  What changes is the end
// of each layer.  There, the MLP hidden vector (4864 values) was handed to
// every CTA -- 38 KB of flagged words polled by each of 148 CTAs -- and each
// CTA then ran its own 6 rows of W_down over the whole vector.  Here:
//
//   S4  RMSNorm(x) -> this CTA's gate/up row pairs -> SwiGLU: the CTA now
//       holds its own ~33 hidden values, and multiplies them right away by
//       the matching ~33 COLUMNS of W_down -- rows of a transposed copy
//       W_downT[layer][4864][896] the engine writes at load time, staged in
//       shared memory one stage ahead like every other weight -- giving a
//       partial 896-vector, published as flagged words (one block per CTA);
//   S5  each CTA sums, for its ~6 residual rows, the partials of all CTAs in
//       CTA order (deterministic), adds them to x and publishes the x words.
//
// So the hidden vector never leaves its CTA, and the hand-off at the end of
// the layer polls ~900 words per CTA instead of 4864.  The weight bytes per
// token are unchanged (W_downT replaces W_down).  The hidden values enter
// the mixed-precision dot as fp16 hi + lo (x = hi + lo, ~22 bits), scaled by
// a power of two when the CTA's largest |value| approaches the fp16 range,
// so no value overflows and the scaling is exact.
//
// Shared memory: per warp 5 weight rows + an O half-row (the LM-head ring's
// sixth row per warp lives in the W_downT region, free by then), the
// W_downT rows of the CTA, the attention scratch and the fp16 hi / lo
// activation vectors.
#pragma once
#include "qwen_mk.cuh"

namespace qmk2 {
using namespace mkc;
using qmk::C;
using qmk::CPR;
using qmk::FC;
using qmk::HD;
using qmk::KVD;
using qmk::LBASE;
using qmk::LSTRIDE;
using qmk::L_DOWN;
using qmk::L_GATEUP;
using qmk::L_INLN;
using qmk::L_OW;
using qmk::L_POST;
using qmk::L_QKVB;
using qmk::L_QKVW;
using qmk::NH;
using qmk::NKV;
using qmk::NL;
using qmk::OFF_COS;
using qmk::OFF_LNF;
using qmk::OFF_SIN;
using qmk::QKV;
using qmk::SPLITS_MAX;
using qmk::THREADS;
using qmk::V;
using qmk::WARPS;

constexpr int HEAD_ROWS = 5;             // per-warp weight rows (S1: 2 QKV rows, S4: <= 5 gate/up rows)
constexpr int WHEAD = HEAD_ROWS * C * 2;  // 8960 B
constexpr int WREG = WHEAD + C;           // + the O half-row: 9856 B per warp
constexpr int LM_G = 3, LM_NB = 2;        // LM head: groups of 3 rows, 2 groups in flight (6 ring rows)
constexpr int MB_HEAD = 0, MB_TAIL = 1, MB_DOWN = 2, MB_LM = 3, NMB = 3 + LM_NB;
constexpr int HID_MAX = 48;               // gate/up pairs per CTA (<= ceil(4864 / 128) = 38)
// Flagged words, laid out so that every 128-byte line is written by ONE
// store instruction of one CTA (a line whose words arrive from several
// stores reaches its pollers later): x | q k v | attention partials | down
// partials.  x: CTA b's residual rows (<= 16) in line b; attention
// partial (head, split): o[64], m, l in 80 words (5 lines); down partials:
// 896 words per CTA.
constexpr int GMAX = 160, XLINE = 16, PW = 80;
constexpr int LL_X = 0, LL_QKV = GMAX * XLINE, LL_PART = LL_QKV + QKV, LL_DP = LL_PART + NH * SPLITS_MAX * PW;
static_assert(LL_DP == SB_MK2_LL_DP, "flagged-word layout");
static_assert(LL_PART % 16 == 0 && LL_DP % 16 == 0 && (C * 8) % 128 == 0 && (PW * 8) % 128 == 0,
              "regions and blocks start on 128-byte lines");
// the CTA (of G) that owns residual row i: the largest b with C*b/G <= i
SB_DEV int x_owner(int i, int G) { return ((i + 1) * G - 1) / C; }

// The dot of 3 rows at independent addresses (the LM-head ring) against the
// fp16 hi / lo activation vectors: as qmk::smem_rows_dot_hl.
SB_DEV void rows3_dot_hl(const uint4 *r0, const uint4 *r1, const uint4 *r2, int nvalid, const uint4 *xh,
                         const uint4 *xl, float (&out)[3]) {
    const uint4 *rows[3] = {r0, r1, r2};
    float ah[3] = {0.f, 0.f, 0.f}, al[3] = {0.f, 0.f, 0.f};
    for (int c = threadIdx.x & 31; c < CPR; c += 32) {
        const uint4 h = xh[c], l = xl[c];
        const unsigned hs[4] = {h.x, h.y, h.z, h.w}, ls[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int r = 0; r < 3; r++)
            if (r < nvalid) {
                const uint4 w = rows[r][c];
                const unsigned ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const unsigned short w0 = ws[j] & 0xffffu, w1 = ws[j] >> 16;
                    ah[r] = qmk::fma_hh(ah[r], w0, (unsigned short)(hs[j] & 0xffffu));
                    al[r] = qmk::fma_hh(al[r], w0, (unsigned short)(ls[j] & 0xffffu));
                    ah[r] = qmk::fma_hh(ah[r], w1, (unsigned short)(hs[j] >> 16));
                    al[r] = qmk::fma_hh(al[r], w1, (unsigned short)(ls[j] >> 16));
                }
            }
    }
#pragma unroll
    for (int r = 0; r < 3; r++) out[r] = ah[r] + al[r];
}

// two flagged words (16-byte aligned pair) with one store
SB_DEV void ll_put2(u64 *p, float a, float b, unsigned e) {
    asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(ll_word(a, e)), "l"(ll_word(b, e))
                 : "memory");
}

// power-of-two scale that keeps |v| * s below 2^14 (1 when it already is):
// exact, and the fp16 hi part cannot overflow
SB_DEV float hid_scale(float mx) {
    if (!(mx >= 16384.0f)) return 1.0f;
    int e;
    frexpf(mx, &e);  // mx = f * 2^e, f in [0.5, 1)
    return ldexpf(1.0f, 14 - e);
}
}  // namespace qmk2

// grid: one CTA per SM (cooperative launch, >= 128 CTAs); block qmk::THREADS;
// dynamic smem: WARPS*WREG + ceil(FC/G)*C*2 + score_cap*4
//               + (32 + WARPS*64 + WARPS + NH*SPLITS_MAX*2)*4 + C*4 bytes.
// raw.aux: W_downT [NL][FC][C] fp16 (rows of W_down's transpose per layer).
extern "C" __global__ void __launch_bounds__(qmk::THREADS, 1) qwen_decode_mk2(const SbMkParams raw) {
    using namespace qmk2;
    const Params p(raw);
    const unsigned short *wdt = reinterpret_cast<const unsigned short *>(raw.aux);
    extern __shared__ __align__(16) unsigned char smem[];
    const int b = blockIdx.x, G = gridDim.x;
    const int dsmax = (FC + G - 1) / G;  // W_downT rows a CTA holds at most
    unsigned char *wbase = smem;
    unsigned char *dsreg = smem + (size_t)WARPS * WREG;
    float *scores = reinterpret_cast<float *>(dsreg + (size_t)dsmax * C * 2);
    float *red = scores + ((p.score_cap + 3) & ~3);  // 32 floats
    float *opart = red + 32;                          // WARPS x HD per-warp partial P.V
    float *ksum = opart + WARPS * HD;                 // WARPS floats
    float *mlv = ksum + WARPS;                        // NH*SPLITS_MAX (m, l) pairs
    float *dpart = opart;  // S5: [rows][G] down partials (opart, ksum, mlv are free then: 1264 floats)
    uint4 *xh4 = reinterpret_cast<uint4 *>(mlv + NH * SPLITS_MAX * 2), *xl4 = xh4 + CPR;
    unsigned *xhw = reinterpret_cast<unsigned *>(xh4), *xlw = reinterpret_cast<unsigned *>(xl4);
    unsigned short *xhs = reinterpret_cast<unsigned short *>(xh4), *xls = reinterpret_cast<unsigned short *>(xl4);
    __shared__ float wmax_s[WARPS], xown[8], gu_s[2 * HID_MAX];
    __shared__ float wgt_s[NH * SPLITS_MAX];  // S3: softmax weight of each (head, split) partial
    __shared__ unsigned hid_hl[HID_MAX];
    __shared__ float qkv_o[8][2];  // S1: this CTA's pair outputs (rows r, r + 32)
    __shared__ unsigned long long best_s;
    __shared__ __align__(8) uint64_t mbar[WARPS][NMB];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    unsigned char *wreg = wbase + (size_t)warp * WREG;
    const uint4 *wreg4 = reinterpret_cast<const uint4 *>(wreg);
    if (sb_step_idle(p.st)) return;  // uniform: every CTA reads the same state
    if (lane == 0)
        for (int i = 0; i < NMB; i++) mbar_init(&mbar[warp][i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    if (p.trace && tid == 0) p.trace[(size_t)b * 256] = globaltimer();  // slot 0: start
    const unsigned seq = p.sync[0];
    auto epoch = [&](int l, int s) { return (seq << 7) | (unsigned)(l * 5 + s + 1); };
    auto stamp = [&](int l, int s, int which) {  // which 0: inputs ready, 1: outputs written
        if (p.trace && tid == 0) p.trace[(size_t)b * 256 + 1 + 2 * (l * 5 + s) + which] = globaltimer();
    };
    // finer stamps inside one layer (slots 243 + k, layer TRACE_L only)
    constexpr int TRACE_L = 12;
    auto xstamp = [&](int l, int k) {
        if (p.trace && tid == 0 && l == TRACE_L) p.trace[(size_t)b * 256 + 243 + k] = globaltimer();
    };
    const int pos = p.st->pos, T = pos + 1;
    const int tok = p.tokens[pos];
    const float eps = 1e-6f;
    const unsigned short *emb = p.w;
    const float *cosT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_COS);
    const float *sinT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_SIN);
    const bool xact = tid < C / 2;  // holds x elements (2 tid, 2 tid + 1) in RMS stages
    u64 *const llx = p.ll + LL_X, *const llqkv = p.ll + LL_QKV;
    u64 *const llpart = p.ll + LL_PART, *const lldp = p.ll + LL_DP;

    // per-CTA shares (static over the step)
    int qp0, qp1, or0, or1, gp0, gp1;
    share(QKV / 2, b, G, qp0, qp1);  // RoPE pairs
    share(C, b, G, or0, or1);        // O rows and this CTA's residual rows
    share(FC, b, G, gp0, gp1);       // gate/up pairs = hidden values = W_downT rows
    const int np = gp1 - gp0, nr = or1 - or0, npairs = qp1 - qp0;
    const int nsplit = max(1, min(min(p.splits, SPLITS_MAX), (T + 63) / 64));
    const int slen = (T + nsplit - 1) / nsplit;

    auto layer_ptr = [&](int l) { return p.w + (LBASE / 2) + (long)l * (LSTRIDE / 2); };
    auto wdt_ptr = [&](int l) { return wdt + ((long)l * FC + gp0) * C; };  // this CTA's W_downT rows

    // L2 prefetch of this CTA's slices of layer l in five pieces (one per stage)
    auto prefetch_piece = [&](int l, int piece) {
        if (l >= NL) return;
        const unsigned short *L = layer_ptr(l);
        const long dbytes = (long)np * C * 2, dhalf = (dbytes / 2) & ~15L;
        switch (piece) {
        case 0:
            for (int pp = qp0; pp < qp1; pp++) {
                const int h = pp / 32, i = pp % 32;
                l2_prefetch_bulk(L + L_QKVW + (long)(h * HD + i) * C, C * 2);
                l2_prefetch_bulk(L + L_QKVW + (long)(h * HD + 32 + i) * C, C * 2);
            }
            prefetch_rows(L + L_OW, C * 2, or0, or1, 1L << 20);
            break;
        case 1: prefetch_rows(L + L_GATEUP, C * 2, gp0, gp1, 1L << 20); break;
        case 2: prefetch_rows(L + L_GATEUP, C * 2, FC + gp0, FC + gp1, 1L << 20); break;
        case 3: l2_prefetch_bulk(wdt_ptr(l), (uint32_t)dhalf); break;
        default: l2_prefetch_bulk(reinterpret_cast<const char *>(wdt_ptr(l)) + dhalf, (uint32_t)(dbytes - dhalf)); break;
        }
    };
    const bool prefetcher = (warp == WARPS - 2 && lane == 0);

    // ---- weight staging (lane 0 issues bulk copies; the warp waits on the slot's mbarrier)
    unsigned phase = 0, pend = 0;
    uint64_t *mb = mbar[warp];
    auto fence_async = [&]() {
        if (lane == 0) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    };
    auto issue_begin = [&](int i, unsigned bytes) {  // lane 0 only
        mbar_expect_tx(&mb[i], bytes);
        pend |= 1u << i;
    };
    auto wait_slot = [&](int i) {
        if (!mbar_wait(&mb[i], (phase >> i) & 1u) && lane == 0) atomicExch(p.err, 2);
        phase ^= 1u << i;
        pend &= ~(1u << i);
    };
    auto copy_s1 = [&](int l) {  // warp w < npairs: pair qp0 + w, rows r, r+32
        if (lane != 0) return;
        const int pp = qp0 + warp;
        const bool has = pp < qp1;
        issue_begin(MB_HEAD, has ? 2 * C * 2 : 0);
        if (has) {
            const int h = pp / 32, i = pp % 32;
            const unsigned short *W = layer_ptr(l) + L_QKVW;
            bulk_g2s(wreg, W + (long)(h * HD + i) * C, C * 2, &mb[MB_HEAD]);
            bulk_g2s(wreg + C * 2, W + (long)(h * HD + 32 + i) * C, C * 2, &mb[MB_HEAD]);
        }
    };
    auto copy_s3 = [&](int l) {  // O rows: warp w -> row or0 + w/2, half w%2 (tail slot)
        if (lane != 0) return;
        const int r = or0 + warp / 2, half = warp % 2;
        issue_begin(MB_TAIL, r < or1 ? C : 0);
        if (r < or1) bulk_g2s(wreg + WHEAD, layer_ptr(l) + L_OW + (long)r * C + half * (C / 2), C, &mb[MB_TAIL]);
    };
    // gate/up rows: CTA row r (pair r/2; gate when even, up when odd) -> warp r % 16, head row r / 16
    const int gu_rows = 2 * np;
    const int gu_nr = max(0, (gu_rows - warp + WARPS - 1) / WARPS);  // this warp's rows (<= 5)
    auto copy_s4_piece = [&](int l, int k) {
        if (lane != 0) return;
        if (k == 0) issue_begin(MB_HEAD, (unsigned)gu_nr * C * 2);
        const unsigned short *W = layer_ptr(l) + L_GATEUP;
        for (int t = 2 * k; t < min(gu_nr, 2 * k + 2); t++) {
            const int r = warp + WARPS * t;
            bulk_g2s(wreg + t * C * 2, W + (long)((r & 1) * FC + gp0 + (r >> 1)) * C, C * 2, &mb[MB_HEAD]);
        }
    };
    // the CTA's whole W_downT slice is ONE bulk copy by warp 15, issued a
    // layer ahead, right after the slice was last read (per-warp copies in
    // the attention stage delayed the CTAs with an attention item)
    uint64_t *mb_ds = &mbar[WARPS - 1][MB_DOWN];
    auto copy_ds_one = [&](int l) {
        if (warp != WARPS - 1 || lane != 0) return;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue_begin(MB_DOWN, (unsigned)np * C * 2);
        bulk_g2s(dsreg, wdt_ptr(l), (unsigned)np * C * 2, mb_ds);
    };
    auto wait_ds = [&]() {
        if (!mbar_wait(mb_ds, (phase >> MB_DOWN) & 1u) && lane == 0) atomicExch(p.err, 2);
        phase ^= 1u << MB_DOWN;
        pend &= ~(1u << MB_DOWN);
    };
    float2 xv = make_float2(0.f, 0.f);
    auto wait_x = [&](unsigned e) {
        bool ok = true;
        if (xact) {  // rows 2 tid and 2 tid + 1, each in its owner's line
            const int i0 = 2 * tid, i1 = i0 + 1;
            int lo0, hi0, lo1, hi1;
            const int b0_ = x_owner(i0, G), b1_ = x_owner(i1, G);
            share(C, b0_, G, lo0, hi0);
            share(C, b1_, G, lo1, hi1);
            const u64 *w0 = llx + b0_ * XLINE + (i0 - lo0), *w1 = llx + b1_ * XLINE + (i1 - lo1);
            for (long spin = 0; ok; spin++) {
                const u64 a = ll_get(w0), c = ll_get(w1);
                if (ll_is(a, e) && ll_is(c, e)) {
                    xv = make_float2(ll_val(a), ll_val(c));
                    break;
                }
                ok = ll_keep_polling(spin, p.err);
            }
        }
        return !__syncthreads_or(!ok);
    };
    bool aborted = false;

    // ---- prologue: this CTA's residual rows start as the embedding
    if (tid < nr) xown[tid] = h2f_ftz(emb[(long)tok * C + or0 + tid]);
    if (prefetcher)
        for (int piece = 0; piece < 5; piece++) prefetch_piece(0, piece);
    fence_async();
    copy_s1(0);
    copy_s3(0);
    copy_ds_one(0);
    if (xact) {
        const unsigned e2 = *reinterpret_cast<const unsigned *>(emb + (long)tok * C + 2 * tid);
        xv = make_float2(h2f_ftz((unsigned short)(e2 & 0xffffu)), h2f_ftz((unsigned short)(e2 >> 16)));
    }
    unsigned gw1 = 0u;
    float b0 = 0.f, b1 = 0.f, cs = 0.f, sn = 0.f;
    const int pp1 = qp0 + warp;
    auto s1_consts = [&](int l) {
        const unsigned short *L = layer_ptr(l);
        gw1 = xact ? *reinterpret_cast<const unsigned *>(L + L_INLN + 2 * tid) : 0u;
        if (pp1 < qp1 && lane == 0) {
            const int h = pp1 / 32, i = pp1 % 32;
            b0 = h2f_ftz(L[L_QKVB + h * HD + i]);
            b1 = h2f_ftz(L[L_QKVB + h * HD + 32 + i]);
            cs = cosT[(long)pos * 32 + i];
            sn = sinT[(long)pos * 32 + i];
        }
    };
    s1_consts(0);

    for (int l = 0; l < NL; l++) {
        const unsigned short *L = layer_ptr(l);
        float *kc = p.kv + (long)l * p.ctx_cap * KVD;
        float *vc = p.kv + (long)(NL + l) * p.ctx_cap * KVD;
        // ================= S1: RMSNorm -> QKV -> RoPE -> q, k, v words
        if (l > 0 && !wait_x(epoch(l - 1, 4))) { aborted = true; break; }
        stamp(l, 0, 0);
        qmk::rms_regs(xv, gw1, xhw, xlw, red, eps);
        __syncthreads();
        xstamp(l, 0);  // S1 norm done
        wait_slot(MB_HEAD);
        __syncwarp();
        xstamp(l, 1);  // S1 rows landed
        if (pp1 < qp1) {
            const int h = pp1 / 32;
            float a[2];
            qmk::smem_rows_dot_hl<2>(wreg4, CPR, 2, xh4, xl4, 0, CPR, 0, a);
            const float a0 = warp_sum(a[0]), a1 = warp_sum(a[1]);
            if (lane == 0) {
                float y0 = __fadd_rn(a0, b0), y1 = __fadd_rn(a1, b1);
                if (h < NH + NKV) {
                    const float o0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                    const float o1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
                    y0 = o0;
                    y1 = o1;
                }
                qkv_o[warp][0] = y0;
                qkv_o[warp][1] = y1;
            }
        }
        __syncthreads();
        // the CTA's q / k / v words (two runs: rows r and r + 32 of its pairs)
        // leave with ONE store instruction (lanes 0 .. 2 npairs - 1 of warp 0)
        if (tid < 2 * npairs) {
            const int w = tid % npairs, which = tid / npairs, pp = qp0 + w;
            const int h = pp / 32, r = h * HD + pp % 32 + 32 * which;
            const float y = qkv_o[w][which];
            ll_put(llqkv + r, y, epoch(l, 0));
            if (h >= NH + NKV) vc[(long)pos * KVD + r - C - KVD] = y;
            else if (h >= NH) kc[(long)pos * KVD + r - C] = y;
        }
        stamp(l, 0, 1);
        // (issued here rather than before the S1 dot: the prefetch instructions
        // of one warp delayed the CTA's S1 barrier, 6 us per token)
        if (prefetcher) prefetch_piece(l + 1, 0);
        // gate/up rows (head slot: S1's rows are consumed) and this layer's
        // W_downT rows stream in while attention runs; a CTA with an
        // attention item issues them after it
        const bool has_item = b < NH * nsplit;
        auto issue_s3_s4 = [&]() {
            fence_async();
            copy_s4_piece(l, 0);
            copy_s4_piece(l, 1);
            if (prefetcher) prefetch_piece(l + 1, 1);
        };
        if (!has_item) issue_s3_s4();
        // ================= S2: attention partials; a warp per position, K and V
        // rows loaded together so one round trip serves scores and P.V.  Each
        // warp keeps its own softmax (max, sum, P.V) and the CTA combines the
        // sixteen of them once: two barriers per item.
        const unsigned e_qkv = epoch(l, 0);
        for (int item = b; item < NH * nsplit; item += G) {
            const int h = item / nsplit, s = item % nsplit, g = h / (NH / NKV);
            const int t0 = s * slen, t1 = min(T, t0 + slen), n = max(0, t1 - t0);
            const u64 *kcur = llqkv + C + g * HD + 2 * lane, *vcur = llqkv + C + KVD + g * HD + 2 * lane;
            if (item != b) __syncthreads();  // a later item: the previous one's readers are done
            float2 kk[4], vv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int t = t0 + warp + WARPS * k;
                kk[k] = vv[k] = make_float2(0.f, 0.f);
                if (t < t1 && t < pos) {
                    kk[k] = __ldcg(reinterpret_cast<const float2 *>(kc + (long)t * KVD + g * HD) + lane);
                    vv[k] = __ldcg(reinterpret_cast<const float2 *>(vc + (long)t * KVD + g * HD) + lane);
                }
            }
            // warps 0, 1, 2 wait for q_h, the current k, the current v at once
            // (one poller per quantity: all sixteen warps on the same hot
            // words slowed their producers' stores).  The hi / lo activation
            // planes are free during this stage and hold them.
            float2 *qkv_s = reinterpret_cast<float2 *>(xh4);
            bool ok = true;
            if (warp == 0 || (t1 == T && warp < 3)) {
                const u64 *src = warp == 0 ? llqkv + h * HD + 2 * lane : (warp == 1 ? kcur : vcur);
                float2 v;
                ok = ll_wait2(src, e_qkv, v.x, v.y, p.err);
                qkv_s[32 * warp + lane] = v;
            }
            if (__syncthreads_or(!ok)) { aborted = true; break; }
            xstamp(l, 2);  // S2 q, k, v arrived (item CTAs)
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
            // positions beyond 64 per item (long contexts): scores via smem, V
            // re-read (the current position's V word is kept from here)
            float2 vpos = make_float2(0.f, 0.f);
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) {
                const int t = t0 + j;
                float2 k2;
                if (t == pos) {
                    k2 = qkv_s[32 + lane];
                    vpos = qkv_s[64 + lane];
                } else {
                    k2 = __ldcg(reinterpret_cast<const float2 *>(kc + (long)t * KVD + g * HD) + lane);
                }
                const float d = warp_sum(fmaf(q2.x, k2.x, q2.y * k2.y)) * 0.125f;
                if (lane == 0) scores[j] = d;
            }
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
                const float2 v2 = t == pos ? vpos
                                           : __ldcg(reinterpret_cast<const float2 *>(vc + (long)t * KVD + g * HD) + lane);
                o.x = fmaf(e, v2.x, o.x);
                o.y = fmaf(e, v2.y, o.y);
            }
            reinterpret_cast<float2 *>(opart + warp * HD)[lane] = o;
            if (lane == 0) {
                ksum[warp] = lsum;
                wmax_s[warp] = wm;
            }
            __syncthreads();
            if (tid < HD) {  // the sixteen warp softmaxes combined: partial (o, m, l) of this item
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
        }
        if (aborted) break;
        stamp(l, 1, 1);
        if (has_item) issue_s3_s4();
        xstamp(l, 3);  // S2 over, next-stage copies issued
        // ================= S3: combine partials -> att; O rows; x += O att
        copy_s4_piece(l, 2);
        if (prefetcher) prefetch_piece(l + 1, 2);
        {
            const unsigned e = epoch(l, 1);
            bool ok = true;
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
            // each (head, split) weight once, not once per output element
            if (tid < NH * nsplit) {
                const int h = tid / nsplit;
                float M = -1e30f;
                for (int s = 0; s < nsplit; s++) M = fmaxf(M, mlv[2 * (h * nsplit + s)]);
                wgt_s[tid] = expf(mlv[2 * tid] - M);
            }
            __syncthreads();
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int d = tid + THREADS * u;
                if (d >= C) break;
                const int h = d / HD;
                float acc = 0.f, Lsum = 0.f;
#pragma unroll
                for (int s = 0; s < SPLITS_MAX; s++) {
                    if (s < nsplit) {
                        const float wgt = wgt_s[h * nsplit + s];
                        Lsum = fmaf(wgt, mlv[2 * (h * nsplit + s) + 1], Lsum);
                        acc = fmaf(wgt, ov[u][s], acc);
                    }
                }
                qmk::split_hl(acc / Lsum, xhs[d], xls[d]);
            }
        }
        __syncthreads();
        xstamp(l, 4);  // S3 combine done
        wait_slot(MB_TAIL);
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            qmk::smem_rows_dot_hl<1>(wreg4 + WHEAD / 16, 0, r < or1 ? 1 : 0, xh4, xl4, half * (CPR / 2),
                                     (half + 1) * (CPR / 2), half * (CPR / 2), a);
            const float y = warp_sum(a[0]);
            if (lane == 0) ksum[warp] = y;
            __syncthreads();
            if (tid < nr) {
                const float xn = __fadd_rn(xown[tid], ksum[2 * tid] + ksum[2 * tid + 1]);
                xown[tid] = xn;
                ll_put(llx + b * XLINE + tid, xn, epoch(l, 2));
            }
        }
        if (l + 1 < NL) {  // the tail slot is read: the next layer's O rows
            fence_async();
            copy_s3(l + 1);
        }
        stamp(l, 2, 1);
        // ================= S4: RMSNorm -> gate/up -> SwiGLU -> this CTA's
        // hidden values -> times their W_downT rows -> down-partial words
        const unsigned gw4 = xact ? *reinterpret_cast<const unsigned *>(L + L_POST + 2 * tid) : 0u;
        if (prefetcher) prefetch_piece(l + 1, 3);
        if (!wait_x(epoch(l, 2))) { aborted = true; break; }
        stamp(l, 3, 0);
        qmk::rms_regs(xv, gw4, xhw, xlw, red, eps);
        __syncthreads();
        wait_slot(MB_HEAD);
        __syncwarp();
        {
            float a[5];
            qmk::smem_rows_dot_hl<5>(wreg4, CPR, gu_nr, xh4, xl4, 0, CPR, 0, a);
#pragma unroll
            for (int t = 0; t < 5; t++) {
                const float d = warp_sum(a[t]);
                if (t < gu_nr && lane == 0) gu_s[warp + WARPS * t] = d;
            }
            __syncthreads();
            xstamp(l, 5);  // S4 gate/up dots done
            // SwiGLU of pair tid (gate row 2 tid, up row 2 tid + 1); warps 0-1
            // also find the largest |value| for the fp16 range scale
            float hv = 0.f;
            if (tid < np) {
                const float ag = gu_s[2 * tid], au = gu_s[2 * tid + 1];
                hv = __fmul_rn(__fdiv_rn(ag, __fadd_rn(1.0f, expf(-ag))), au);
            }
            if (warp < 2) {
                float mx = fabsf(hv);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(SB_FULL, mx, o));
                if (lane == 0) wmax_s[warp] = mx;
            }
            __syncthreads();
            const float hs = hid_scale(fmaxf(wmax_s[0], wmax_s[1]));
            if (tid < np) {
                unsigned short h, lo;
                qmk::split_hl(hv * hs, h, lo);
                hid_hl[tid] = h | ((unsigned)lo << 16);
            }
            wait_ds();
            __syncthreads();
            xstamp(l, 6);  // S4 down rows landed, hidden values split
            if (tid < C / 2) {  // rows 2 tid, 2 tid + 1 of the down product over this CTA's hidden values
                float a0h = 0.f, a0l = 0.f, a1h = 0.f, a1l = 0.f;
                for (int j = 0; j < np; j++) {
                    const unsigned w2 = reinterpret_cast<const unsigned *>(dsreg + (size_t)j * C * 2)[tid];
                    const unsigned hl = hid_hl[j];
                    const unsigned short w0 = w2 & 0xffffu, w1 = w2 >> 16, hh = hl & 0xffffu, hl2 = hl >> 16;
                    a0h = qmk::fma_hh(a0h, w0, hh);
                    a0l = qmk::fma_hh(a0l, w0, hl2);
                    a1h = qmk::fma_hh(a1h, w1, hh);
                    a1l = qmk::fma_hh(a1l, w1, hl2);
                }
                const float inv = 1.0f / hs;  // a power of two: exact
                ll_put2(lldp + (long)b * C + 2 * tid, (a0h + a0l) * inv, (a1h + a1l) * inv, epoch(l, 3));
            }
        }
        stamp(l, 3, 1);
        if (l + 1 < NL) s1_consts(l + 1);  // the loads' latency hides in the S5 wait
        // ================= S5: this CTA's residual rows += the down partials
        // of all CTAs (summed in CTA order) -> x words
        if (prefetcher) prefetch_piece(l + 1, 4);
        {
            const unsigned e = epoch(l, 3);
            const int nitems = nr * G;  // (producer q, row r) pairs, q-major
            bool ok = true;
            for (long spin = 0; ok; spin++) {
                bool all = true;
                for (int k = tid; k < nitems; k += THREADS) {
                    const int q = k / nr, r = k % nr;
                    const u64 wv = ll_get(lldp + (long)q * C + or0 + r);
                    if (ll_is(wv, e)) dpart[r * G + q] = ll_val(wv);
                    else all = false;
                }
                if (all) break;
                ok = ll_keep_polling(spin, p.err);
            }
            if (__syncthreads_or(!ok)) { aborted = true; break; }
            stamp(l, 4, 0);
            if (l + 1 < NL) copy_ds_one(l + 1);  // every warp has read the slice
            // the row sums meet in shared memory and one warp stores all of
            // this CTA's x words with one instruction: words of one line
            // written by several warps at different times reached the
            // pollers ~1.5 us later
            if (warp < nr) {
                float sum = 0.f;
                for (int q = lane; q < G; q += 32) sum += dpart[warp * G + q];
                sum = warp_sum(sum);
                if (lane == 0) wmax_s[warp] = sum;
            }
            __syncthreads();
            if (tid < nr) {
                const float xn = __fadd_rn(xown[tid], wmax_s[tid]);
                xown[tid] = xn;
                // test hook: the stalled CTA withholds its layer-0 outputs
                if (!(p.test_stall == b + 1 && l == 0)) ll_put(llx + b * XLINE + tid, xn, epoch(l, 4));
            }
        }
        stamp(l, 4, 1);
        if (l + 1 < NL) {
            fence_async();
            copy_s1(l + 1);
            xstamp(l, 7);  // S5 next S1 rows issued
        }
    }
    if (aborted) {
        if (lane == 0)
            for (int i = 0; i < NMB; i++)
                if ((pend >> i) & 1u) mbar_wait(&mb[i], (phase >> i) & 1u);
        return;
    }
    // ================= LM head + argmax (ring rows 0-4 in the warp's head
    // slot, row 5 in the W_downT region, which every warp of this CTA has
    // finished reading: the S5 barrier above)
    if (p.with_logits) {
        int v0, v1;
        share(V, b, G, v0, v1);
        const int nrow = max(0, (v1 - v0 - warp + WARPS - 1) / WARPS);
        const int ngrp = (nrow + LM_G - 1) / LM_G;
        auto ring_row = [&](int rr) -> unsigned char * {
            return rr < HEAD_ROWS ? wreg + rr * C * 2 : dsreg + (size_t)warp * C * 2;
        };
        auto issue_grp = [&](int k) {  // lane 0
            const int slot = k % LM_NB, j0 = k * LM_G, nj = min(LM_G, nrow - j0);
            issue_begin(MB_LM + slot, (unsigned)nj * C * 2);
            for (int j = 0; j < nj; j++)
                bulk_g2s(ring_row(slot * LM_G + j), emb + (long)(v0 + warp + WARPS * (j0 + j)) * C, C * 2,
                         &mb[MB_LM + slot]);
        };
        fence_async();
        if (lane == 0)
            for (int k = 0; k < min(LM_NB, ngrp); k++) issue_grp(k);
        const unsigned gwf = xact ? *reinterpret_cast<const unsigned *>(p.w + OFF_LNF / 2 + 2 * tid) : 0u;
        if (tid == 0) best_s = 0ull;
        if (!wait_x(epoch(NL - 1, 4))) {
            if (lane == 0)
                for (int i = 0; i < NMB; i++)
                    if ((pend >> i) & 1u) mbar_wait(&mb[i], (phase >> i) & 1u);
            return;
        }
        qmk::rms_regs(xv, gwf, xhw, xlw, red, eps);
        __syncthreads();
        unsigned long long best = 0ull;
        for (int k = 0; k < ngrp; k++) {
            const int slot = k % LM_NB, j0 = k * LM_G, nj = min(LM_G, nrow - j0);
            wait_slot(MB_LM + slot);
            __syncwarp();
            float a[LM_G];
            rows3_dot_hl(reinterpret_cast<const uint4 *>(ring_row(slot * LM_G)),
                         reinterpret_cast<const uint4 *>(ring_row(slot * LM_G + 1)),
                         reinterpret_cast<const uint4 *>(ring_row(slot * LM_G + 2)), nj, xh4, xl4, a);
#pragma unroll
            for (int j = 0; j < LM_G; j++) {
                const float dotv = warp_sum(a[j]);
                if (j < nj) {
                    const int r = v0 + warp + WARPS * (j0 + j);
                    if (lane == 0) p.logits[r] = dotv;
                    const unsigned long long key = argmax_key(dotv, r);
                    best = key > best ? key : best;
                }
            }
            __syncwarp();
            if (k + LM_NB < ngrp && lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_grp(k + LM_NB);
            }
        }
        if (lane == 0 && best) atomicMax(&best_s, best);
        __syncthreads();
        if (tid == 0) {
            if (best_s) atomicMax(&p.st->key, best_s);
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.sync + 1) : "memory");
        }
        if (p.trace && tid == 0) p.trace[(size_t)b * 256 + 1 + 2 * 120] = globaltimer();
        if (b != 0 || tid != 0) return;
        for (long spin = 0; ld_acquire(p.sync + 1) < (unsigned)G; spin++)
            if (!ll_keep_polling(spin, p.err)) return;
        p.sync[1] = 0u;
    } else if (b != 0 || tid != 0) {
        return;
    }
    // ================= finalize (one thread of CTA 0), as sb_finalize
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
