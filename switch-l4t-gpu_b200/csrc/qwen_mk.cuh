// qwen_mk.cuh -- the whole Qwen2.5-0.5B decode step as ONE persistent,
// cooperatively launched kernel (one CTA per SM).
//
// Why: a decode step is ~120 dependent matvec stages; as separate kernels
// each pays launch, ramp-up and a chain of dependent global round trips
// (measured ~6-13 us per kernel).  Here the stages run back to back inside
// one launch and the weights -- which never depend on the activations --
// are fetched ahead of time:
//   * each warp copies its rows of the NEXT stage into its own shared-memory
//     region with TMA bulk copies as soon as its current rows are consumed,
//     so the copies land while the stage's inputs are still being produced;
//   * one lane issues L2 bulk prefetches of this CTA's slice of the next
//     layer (~200 KB per CTA, ~30 MB in total) in five pieces, so HBM streams
//     underneath the dependency chain.
//
// Stage hand-off without grid barriers: every activation value a stage
// produces is stored as one 8-byte word (float bits | epoch << 32) with a
// single relaxed 64-bit store; the consumer polls exactly the words it needs
// until their epoch is the current one.  A 64-bit aligned access is
// single-copy atomic, so a word whose epoch matches carries its value: no
// fence, no counter, one round trip from producer store to consumer load.
// Epoch = (step sequence number << 7) | (layer * 5 + stage + 1); the
// sequence number advances once per step, so stale words never match.  A
// buffer is rewritten only after every consumer of its previous contents
// has finished (each stage needs ALL outputs of the one before, which in
// turn were computed from the buffer), so one buffer per quantity suffices.
//
// Stages per layer (each CTA owns a contiguous block of rows of every matrix):
//   S1 RMSNorm(x) -> QKV rows (RoPE pairs) + bias + RoPE -> q, k, v words
//      (and k, v into the KV cache for later steps)
//   S2 attention partials: (head, T-split) items, one per CTA; the cached
//      K/V rows are loaded before q arrives
//   S3 combine partials -> att; O rows; x += O att  -> x words (own rows)
//   S4 RMSNorm(x) -> gate/up row pairs -> SwiGLU -> hid words
//   S5 down rows (split-K over warp pairs); x += down hid -> x words
// then final RMSNorm -> LM head rows (three-row groups per warp, two groups
// of bulk copies in flight) -> logits +
// argmax; CTA 0 counts the arrivals and finalises the step (next token,
// position, sequence number).
//
// Waits are bounded: after LL_SPIN_LIMIT polls the kernel sets *err, drains
// its own bulk copies and returns; the host reports the error.
#pragma once
#include "sb_attn.cuh"
#include "sb_finalize.cuh"
#include "sb_gemv.cuh"
#include "sb_mk_common.cuh"
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
constexpr int WHEAD = 6 * C * 2;      // per-warp head slot: 6 rows of 896 fp16 (S1, S4, S5, LM head)
constexpr int WREG = WHEAD + C;       // + tail slot for the O half-row (896 B): 11648 B per warp
constexpr int LM_G = 3;               // LM-head rows a warp reduces together (one group)
constexpr int LM_NB = 2;              // LM-head groups in flight per warp (2 x 3 rows = the head slot)
constexpr int SPLITS_MAX = SB_MK_SPLITS_MAX;
constexpr int PW = HD + 2;            // words per attention partial: o[64], m, l
// flagged-word layout (u64 words)
constexpr int LL_X = 0, LL_QKV = LL_X + C, LL_HID = LL_QKV + QKV, LL_PART = LL_HID + FC;
constexpr int LL_WORDS = LL_PART + NH * SPLITS_MAX * PW;
static_assert(LL_WORDS == SB_MK_LL_WORDS, "flagged-word layout");
static_assert(LL_QKV % 2 == 0 && LL_HID % 2 == 0 && LL_PART % 2 == 0 && PW % 2 == 0, "pairs stay 16-byte aligned");
constexpr int HID_PAIRS = (FC / 2 + THREADS - 1) / THREADS;  // hid word pairs per thread (5)
static_assert(C >= THREADS && NH * SPLITS_MAX <= THREADS,
              "the combine polls each (m, l) pair with the o words of dim tid");

using namespace mkc;

// R rows at base + r*stride (uint4 units) against the split x planes,
// chunk range [c0, c1) (row data starts at chunk row_c0); each x chunk is
// read once for all rows.  Rows >= nvalid are skipped.  Returns per-lane
// partial sums (not yet reduced over the warp).
template <int R>
SB_DEV void smem_rows_dot(const uint4 *base, int stride, int nvalid, const float4 *lo, const float4 *hi, int c0,
                          int c1, int row_c0, float (&out)[R]) {
    unsigned long long acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0ull;
    for (int c = c0 + (threadIdx.x & 31); c < c1; c += 32) {
        const float4 a = lo[c], bq = hi[c];
#pragma unroll
        for (int r = 0; r < R; r++)
            if (r < nvalid) acc[r] = dot8_h_f2(base[r * stride + c - row_c0], a, bq, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < R; r++) out[r] = f2_sum(acc[r]);
}

// The same dot with x given as two fp16 vectors, x = xh + xl (xh = fp16(x),
// xl = fp16(x - xh): ~22 bits of x), on sm_100's mixed-precision FMA
// (fma.rn.f32.f16: exact f16 x f16 product, one FP32 rounding), which needs
// no fp16 -> fp32 conversions -- the limit of the form above.  Two FP32
// accumulators per row (xh terms, xl terms).  Used where x is a norm or an
// attention output (|x| far below the fp16 range), not for the MLP hidden
// vector.  Weights are pre-flushed, so no subnormal handling here.
SB_DEV float fma_hh(float acc, unsigned short a, unsigned short b) {
    asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(a), "h"(b));
    return acc;
}
template <int R>
SB_DEV void smem_rows_dot_hl(const uint4 *base, int stride, int nvalid, const uint4 *xh, const uint4 *xl, int c0,
                             int c1, int row_c0, float (&out)[R]) {
    float ah[R], al[R];
#pragma unroll
    for (int r = 0; r < R; r++) ah[r] = al[r] = 0.f;
    for (int c = c0 + (threadIdx.x & 31); c < c1; c += 32) {
        const uint4 h = xh[c], l = xl[c];
        const unsigned hs[4] = {h.x, h.y, h.z, h.w}, ls[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int r = 0; r < R; r++)
            if (r < nvalid) {
                const uint4 w = base[r * stride + c - row_c0];
                const unsigned ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const unsigned short w0 = ws[j] & 0xffffu, w1 = ws[j] >> 16;
                    ah[r] = fma_hh(ah[r], w0, (unsigned short)(hs[j] & 0xffffu));
                    al[r] = fma_hh(al[r], w0, (unsigned short)(ls[j] & 0xffffu));
                    ah[r] = fma_hh(ah[r], w1, (unsigned short)(hs[j] >> 16));
                    al[r] = fma_hh(al[r], w1, (unsigned short)(ls[j] >> 16));
                }
            }
    }
#pragma unroll
    for (int r = 0; r < R; r++) out[r] = ah[r] + al[r];
}
SB_DEV void split_hl(float v, unsigned short &h, unsigned short &l) {
    const __half hv = __float2half_rn(v);
    h = __half_as_ushort(hv);
    l = __half_as_ushort(__float2half_rn(v - __half2float(hv)));
}

// Element i of a K-vector lives in plane (i%8)<4 ? lo : hi, float (i/8)*4 + i%4.
SB_DEV float *plane_elem(float4 *lo, float4 *hi, int i) {
    return reinterpret_cast<float *>((i & 7) < 4 ? lo : hi) + (i >> 3) * 4 + (i & 3);
}

// RMSNorm from registers: thread t < C/2 holds elements (2t, 2t+1) of x in
// xv and the two fp16 gains in gw (packed); writes x*inv*g into the split
// planes.
SB_DEV void rms_regs(float2 xv, unsigned gw, unsigned *xh, unsigned *xl, float *red, float eps) {
    const int t = threadIdx.x;
    const bool act = t < C / 2;
    float s = act ? fmaf(xv.x, xv.x, xv.y * xv.y) : 0.0f;
    s = block_sum1(s, red, 0);
    const float inv = 1.0f / sqrtf(__fdiv_rn(s, (float)C) + eps);
    if (act) {
        const float g0 = h2f_ftz((unsigned short)(gw & 0xffffu)), g1 = h2f_ftz((unsigned short)(gw >> 16));
        unsigned short h0, l0, h1, l1;
        split_hl(__fmul_rn(__fmul_rn(xv.x, inv), g0), h0, l0);
        split_hl(__fmul_rn(__fmul_rn(xv.y, inv), g1), h1, l1);
        xh[t] = h0 | ((unsigned)h1 << 16);  // elements 2t, 2t + 1
        xl[t] = l0 | ((unsigned)l1 << 16);
    }
}

}  // namespace qmk

// grid: one CTA per SM (cooperative launch, >= 128 CTAs); block qmk::THREADS;
// dynamic smem: FC*4 + WARPS*WREG + score_cap*4
//               + (32 + WARPS*64 + WARPS + NH*SPLITS_MAX*2)*4 + C*4 bytes.
extern "C" __global__ void __launch_bounds__(qmk::THREADS, 1) qwen_decode_mk(const SbMkParams raw) {
    using namespace qmk;
    const Params p(raw);
    extern __shared__ __align__(16) unsigned char smem[];
    // layout: x planes (FC floats) | weight regions (WARPS * WREG) | scores | small
    float4 *xlo = reinterpret_cast<float4 *>(smem);
    float4 *xhi = xlo + CPR_D;  // planes sized for K = FC
    unsigned char *wbase = smem + (size_t)FC * 4;
    float *scores = reinterpret_cast<float *>(wbase + (size_t)WARPS * WREG);
    // float2/float4 accesses follow: keep every region 16-byte aligned
    float *red = scores + ((p.score_cap + 3) & ~3);  // 32 floats
    float *opart = red + 32;                          // WARPS x HD per-warp partial P.V
    float *ksum = opart + WARPS * HD;                 // WARPS floats: split-K partials / per-warp softmax sums
    float *mlv = ksum + WARPS;                        // NH*SPLITS_MAX (m, l) pairs of the partials
    // K = C activations as fp16 hi / lo vectors (S1, S3, S4 and LM-head dots)
    uint4 *xh4 = reinterpret_cast<uint4 *>(mlv + NH * SPLITS_MAX * 2), *xl4 = xh4 + CPR;
    unsigned *xhw = reinterpret_cast<unsigned *>(xh4), *xlw = reinterpret_cast<unsigned *>(xl4);
    unsigned short *xhs = reinterpret_cast<unsigned short *>(xh4), *xls = reinterpret_cast<unsigned short *>(xl4);
    __shared__ float wmax_s[WARPS], xown[8], gu_s[96];
    __shared__ unsigned long long best_s;
    __shared__ __align__(8) uint64_t mbar[WARPS][2 + LM_NB];

    const int b = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    unsigned char *wreg = wbase + (size_t)warp * WREG;
    const uint4 *wreg4 = reinterpret_cast<const uint4 *>(wreg);
    if (sb_step_idle(p.st)) return;  // uniform: every CTA reads the same state
    if (lane == 0)
        for (int i = 0; i < 2 + LM_NB; i++) mbar_init(&mbar[warp][i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    if (p.trace && tid == 0) p.trace[(size_t)b * 256] = globaltimer();  // slot 0: start
    const unsigned seq = p.sync[0];
    auto epoch = [&](int l, int s) { return (seq << 7) | (unsigned)(l * 5 + s + 1); };
    auto stamp = [&](int l, int s, int which) {  // which 0: inputs ready, 1: outputs written
        if (p.trace && tid == 0) p.trace[(size_t)b * 256 + 1 + 2 * (l * 5 + s) + which] = globaltimer();
    };
    const int pos = p.st->pos, T = pos + 1;
    const int tok = p.tokens[pos];
    const float eps = 1e-6f;
    const unsigned short *emb = p.w;
    const float *cosT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_COS);
    const float *sinT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_SIN);
    const bool xact = tid < C / 2;  // holds x elements (2 tid, 2 tid + 1) in RMS stages
    u64 *const llx = p.ll + LL_X, *const llqkv = p.ll + LL_QKV, *const llhid = p.ll + LL_HID;
    u64 *const llpart = p.ll + LL_PART;

    // per-CTA shares (static over the step)
    int qp0, qp1, or0, or1, gp0, gp1;
    share(QKV / 2, b, G, qp0, qp1);  // RoPE pairs
    share(C, b, G, or0, or1);        // O rows and down rows (this CTA's residual rows)
    share(FC, b, G, gp0, gp1);       // gate/up pairs
    // attention T-splits: ~64 positions per item (16 warps each hold up to
    // 4 positions' K/V in registers), at most p.splits per head.  Fewer,
    // fuller items leave S3 fewer partials to poll: 442.6 against 445.3 us
    // per token with ~48 (32: 454.0).
    const int nsplit = max(1, min(min(p.splits, SPLITS_MAX), (T + 63) / 64));
    const int slen = (T + nsplit - 1) / nsplit;

    auto layer_ptr = [&](int l) { return p.w + (LBASE / 2) + (long)l * (LSTRIDE / 2); };

    // L2 prefetch of this CTA's slices of layer l, in five pieces of ~40 KB
    // (one per stage) so the weight stream is spread evenly over the layer
    // instead of bursting in front of the latency-critical activation traffic.
    auto prefetch_piece = [&](int l, int piece) {
        if (l >= NL) return;
        const unsigned short *L = layer_ptr(l);
        const int dmid = or0 + (or1 - or0) / 2;
        switch (piece) {
        case 0:
            for (int pp = qp0; pp < qp1; pp++) {  // QKV pair rows (few)
                const int h = pp / 32, i = pp % 32;
                l2_prefetch_bulk(L + L_QKVW + (long)(h * HD + i) * C, C * 2);
                l2_prefetch_bulk(L + L_QKVW + (long)(h * HD + 32 + i) * C, C * 2);
            }
            prefetch_rows(L + L_OW, C * 2, or0, or1, 1L << 20);
            break;
        case 1: prefetch_rows(L + L_GATEUP, C * 2, gp0, gp1, 1L << 20); break;
        case 2: prefetch_rows(L + L_GATEUP, C * 2, FC + gp0, FC + gp1, 1L << 20); break;
        case 3: prefetch_rows(L + L_DOWN, (long)FC * 2, or0, dmid, 1L << 20); break;
        default: prefetch_rows(L + L_DOWN, (long)FC * 2, dmid, or1, 1L << 20); break;
        }
    };
    const bool prefetcher = (warp == WARPS - 2 && lane == 0);

    // ---- weight staging into the warp's region by TMA bulk copies (lane 0
    // issues; the warp waits on the slot's mbarrier before reading)
    // mbar[warp][0]: head slot (S1, S4, S5 rows); [1]: tail slot (O half-row);
    // [2 + k]: LM-head ring slot k.  `phase` bit i = parity to wait for next;
    // `pend` bit i (lane 0) = a copy into slot i has not been waited for.
    unsigned phase = 0, pend = 0;
    uint64_t *mb = mbar[warp];
    // Lane 0 orders the warp's earlier generic accesses of its region before
    // the async-proxy writes of the copies it issues next (once per batch).
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
        issue_begin(0, has ? 2 * C * 2 : 0);
        if (has) {
            const int h = pp / 32, i = pp % 32;
            const unsigned short *W = layer_ptr(l) + L_QKVW;
            bulk_g2s(wreg, W + (long)(h * HD + i) * C, C * 2, &mb[0]);
            bulk_g2s(wreg + C * 2, W + (long)(h * HD + 32 + i) * C, C * 2, &mb[0]);
        }
    };
    auto copy_s3 = [&](int l) {  // O rows: warp w -> row or0 + w/2, half w%2 (tail slot)
        if (lane != 0) return;
        const int r = or0 + warp / 2, half = warp % 2;
        issue_begin(1, r < or1 ? C : 0);
        if (r < or1) bulk_g2s(wreg + WHEAD, layer_ptr(l) + L_OW + (long)r * C + half * (C / 2), C, &mb[1]);
    };
    // gate/up rows: the CTA's 2*(gp1-gp0) rows r (pair r/2; gate when r is
    // even, up when odd) go to warp r % 16, slot row r / 16 -- at most 5 rows
    // a warp (a pair-per-warp split left one warp with 6 rows when the CTA
    // owns 33 pairs).  The byte count is announced with the first piece, then
    // two slot rows are issued per stage (S1, S2, S3) to spread the traffic.
    const int gu_rows = 2 * (gp1 - gp0);
    const int gu_nr = max(0, (gu_rows - warp + WARPS - 1) / WARPS);  // this warp's rows (<= 5)
    auto copy_s4_piece = [&](int l, int k) {
        if (lane != 0) return;
        if (k == 0) issue_begin(0, (unsigned)gu_nr * C * 2);
        const unsigned short *W = layer_ptr(l) + L_GATEUP;
        for (int t = 2 * k; t < min(gu_nr, 2 * k + 2); t++) {
            const int r = warp + WARPS * t;
            bulk_g2s(wreg + t * C * 2, W + (long)((r & 1) * FC + gp0 + (r >> 1)) * C, C * 2, &mb[0]);
        }
    };
    auto copy_s5 = [&](int l) {  // down rows: warp w -> row or0 + w/2, half w%2 of K
        if (lane != 0) return;
        const int r = or0 + warp / 2, half = warp % 2;
        issue_begin(0, r < or1 ? FC : 0);
        if (r < or1) bulk_g2s(wreg, layer_ptr(l) + L_DOWN + (long)r * FC + half * (FC / 2), FC, &mb[0]);
    };
    // Split-K (2 warps per row) reduction + residual update of this CTA's
    // rows, published as x words of epoch e.
    auto resid_update = [&](float a, unsigned e) {
        if (lane == 0) ksum[warp] = a;
        __syncthreads();
        if (tid < or1 - or0) {
            const float y = ksum[2 * tid] + ksum[2 * tid + 1];
            const float xn = __fadd_rn(xown[tid], y);
            xown[tid] = xn;
            // test hook: the stalled CTA withholds its layer-0 outputs
            if (!(p.test_stall == b + 1 && e == epoch(0, 4))) ll_put(llx + or0 + tid, xn, e);
        }
    };
    // x words of epoch e -> xv (thread t < C/2: elements 2t, 2t+1); uniform
    // result: false when this or another CTA gave up.
    float2 xv = make_float2(0.f, 0.f);
    auto wait_x = [&](unsigned e) {
        bool ok = true;
        if (xact) ok = ll_wait2(llx + 2 * tid, e, xv.x, xv.y, p.err);
        return !__syncthreads_or(!ok);
    };
    bool aborted = false;

    // ---- prologue: this CTA's residual rows start as the embedding
    if (tid < or1 - or0) xown[tid] = h2f_ftz(emb[(long)tok * C + or0 + tid]);
    if (prefetcher)
        for (int piece = 0; piece < 5; piece++) prefetch_piece(0, piece);
    fence_async();
    copy_s1(0);
    copy_s3(0);  // O rows: one layer ahead from here on
    // layer-0 S1 input: the embedding row (constant: nothing to wait for)
    if (xact) {
        const unsigned e2 = *reinterpret_cast<const unsigned *>(emb + (long)tok * C + 2 * tid);
        xv = make_float2(h2f_ftz((unsigned short)(e2 & 0xffffu)), h2f_ftz((unsigned short)(e2 >> 16)));
    }
    // S1 constants of layer l (norm gains, this warp's bias pair, RoPE cos/sin)
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
        rms_regs(xv, gw1, xhw, xlw, red, eps);
        __syncthreads();
        // (An L2 prefetch of the LM-head rows during the last layers measured
        // 10 us per token slower: it competes with those layers' weights.)
        if (prefetcher) prefetch_piece(l + 1, 0);
        wait_slot(0);
        __syncwarp();
        if (pp1 < qp1) {
            const int h = pp1 / 32, i = pp1 % 32;
            const int r0 = h * HD + i, r1 = r0 + 32;
            float a[2];
            smem_rows_dot_hl<2>(wreg4, CPR, 2, xh4, xl4, 0, CPR, 0, a);
            const float a0 = warp_sum(a[0]), a1 = warp_sum(a[1]);
            if (lane == 0) {
                float y0 = __fadd_rn(a0, b0), y1 = __fadd_rn(a1, b1);
                if (h < NH + NKV) {
                    const float o0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                    const float o1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
                    y0 = o0;
                    y1 = o1;
                }
                const unsigned e = epoch(l, 0);
                ll_put(llqkv + r0, y0, e);
                ll_put(llqkv + r1, y1, e);
                if (h >= NH + NKV) { vc[(long)pos * KVD + r0 - C - KVD] = y0; vc[(long)pos * KVD + r1 - C - KVD] = y1; }
                else if (h >= NH) { kc[(long)pos * KVD + r0 - C] = y0; kc[(long)pos * KVD + r1 - C] = y1; }
            }
        }
        stamp(l, 0, 1);
        // O rows (tail slot) and two gate/up pairs (head slot: S1's rows are
        // consumed) stream in while attention runs.  A CTA with an attention
        // item issues them after it: issuing bulk copies stalls the issuing
        // lanes for ~1.5 us, and the item is on the critical path.
        const bool has_item = b < NH * nsplit;
        auto issue_s3_s4 = [&]() {
            fence_async();
            copy_s4_piece(l, 0);
            copy_s4_piece(l, 1);
            if (prefetcher) prefetch_piece(l + 1, 1);
        };
        if (!has_item) issue_s3_s4();
        // ================= S2: attention partials; a warp per position, K and V
        // rows loaded together so one round trip serves scores and P.V
        const unsigned e_qkv = epoch(l, 0);
        for (int item = b; item < NH * nsplit; item += G) {
            const int h = item / nsplit, s = item % nsplit, g = h / (NH / NKV);
            const int t0 = s * slen, t1 = min(T, t0 + slen), n = max(0, t1 - t0);
            const u64 *kcur = llqkv + C + g * HD + 2 * lane, *vcur = llqkv + C + KVD + g * HD + 2 * lane;
            __syncthreads();  // the previous item's readers of opart are done
            // each warp keeps up to 4 positions' K and V rows in registers;
            // cached positions (< pos) are requested before q is awaited
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
            // one warp waits for q_h and (when this item holds pos) the current
            // k, v rows and shares them through shared memory: sixteen warps
            // polling the same hot words slow down their producers' stores
            float2 *qkv_s = reinterpret_cast<float2 *>(opart);  // q | k | v pairs (opart is free here)
            bool ok = true;
            if (warp == 0) {
                float2 v;
                ok = ll_wait2(llqkv + h * HD + 2 * lane, e_qkv, v.x, v.y, p.err);
                qkv_s[lane] = v;
                if (t1 == T) {
                    ok = ok && ll_wait2(kcur, e_qkv, v.x, v.y, p.err);
                    qkv_s[32 + lane] = v;
                    ok = ok && ll_wait2(vcur, e_qkv, v.x, v.y, p.err);
                    qkv_s[64 + lane] = v;
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
            if (lane == 0) wmax_s[warp] = wm;
            if (__syncthreads_or(!ok)) { aborted = true; break; }
            float m = -1e30f;
#pragma unroll
            for (int w = 0; w < WARPS; w++) m = fmaxf(m, wmax_s[w]);
            float lsum = 0.f;
            float2 o = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (warp + WARPS * k < n) {
                    const float e = expf(sc[k] - m);
                    lsum += e;
                    o.x = fmaf(e, vv[k].x, o.x);
                    o.y = fmaf(e, vv[k].y, o.y);
                }
            }
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) {
                const int t = t0 + j;
                const float e = expf(scores[j] - m);
                lsum += e;
                const float2 v2 = t == pos ? vpos
                                           : __ldcg(reinterpret_cast<const float2 *>(vc + (long)t * KVD + g * HD) + lane);
                o.x = fmaf(e, v2.x, o.x);
                o.y = fmaf(e, v2.y, o.y);
            }
            reinterpret_cast<float2 *>(opart + warp * HD)[lane] = o;
            if (lane == 0) ksum[warp] = lsum;
            __syncthreads();
            if (tid < HD) {
                float acc = 0.f;
#pragma unroll
                for (int w = 0; w < WARPS; w++) acc += opart[w * HD + tid];
                u64 *pw = llpart + (long)(h * SPLITS_MAX + s) * PW;
                const unsigned e = epoch(l, 1);
                ll_put(pw + tid, acc, e);
                if (tid == 0) {
                    float ls = 0.f;
#pragma unroll
                    for (int w = 0; w < WARPS; w++) ls += ksum[w];
                    ll_put(pw + HD, m, e);
                    ll_put(pw + HD + 1, ls, e);
                }
            }
            __syncthreads();
        }
        if (aborted) break;
        stamp(l, 1, 1);
        if (has_item) issue_s3_s4();
        // ================= S3: combine partials -> att; O rows; x += O att
        copy_s4_piece(l, 2);
        if (prefetcher) prefetch_piece(l + 1, 2);
        {
            const unsigned e = epoch(l, 1);
            bool ok = true;
            // this thread's (m, l) pair (item tid < NH*nsplit <= THREADS) is
            // polled together with its o words below
            const u64 *mlw = llpart + (long)((tid / nsplit) * SPLITS_MAX + tid % nsplit) * PW + HD;
            bool ml_done = tid >= NH * nsplit;
            // the o words of this thread's dims d = tid and tid + THREADS,
            // all splits requested before any is checked
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
                split_hl(acc / Lsum, xhs[d], xls[d]);
            }
        }
        __syncthreads();
        wait_slot(1);  // the O half-row (the gate/up rows may still be landing)
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            smem_rows_dot_hl<1>(wreg4 + WHEAD / 16, 0, r < or1 ? 1 : 0, xh4, xl4, half * (CPR / 2), (half + 1) * (CPR / 2),
                             half * (CPR / 2), a);
            resid_update(warp_sum(a[0]), epoch(l, 2));
        }
        if (l + 1 < NL) {  // the tail slot is read: the next layer's O rows, a layer
            fence_async();   // ahead (-3 us per token; for GPT-2 the same measured slower)
            copy_s3(l + 1);
        }
        stamp(l, 2, 1);
        // ================= S4: RMSNorm -> gate/up -> SwiGLU -> hid words
        const unsigned gw4 = xact ? *reinterpret_cast<const unsigned *>(L + L_POST + 2 * tid) : 0u;
        if (prefetcher) prefetch_piece(l + 1, 3);
        if (!wait_x(epoch(l, 2))) { aborted = true; break; }
        stamp(l, 3, 0);
        rms_regs(xv, gw4, xhw, xlw, red, eps);
        __syncthreads();
        wait_slot(0);
        __syncwarp();
        {
            float a[5];
            smem_rows_dot_hl<5>(wreg4, CPR, gu_nr, xh4, xl4, 0, CPR, 0, a);
#pragma unroll
            for (int t = 0; t < 5; t++) {
                const float d = warp_sum(a[t]);
                if (t < gu_nr && lane == 0) gu_s[warp + WARPS * t] = d;
            }
            __syncthreads();
            if (tid < gp1 - gp0) {  // SwiGLU of pair tid: gate row 2 tid, up row 2 tid + 1
                const float ag = gu_s[2 * tid], au = gu_s[2 * tid + 1];
                ll_put(llhid + gp0 + tid, __fmul_rn(__fdiv_rn(ag, __fadd_rn(1.0f, expf(-ag))), au), epoch(l, 3));
            }
        }
        stamp(l, 3, 1);
        fence_async();
        copy_s5(l);
        // ================= S5: down rows (split-K over warp pairs); x += down hid
        if (prefetcher) prefetch_piece(l + 1, 4);
        {
            // hid words into the planes: every pair this thread owns is
            // requested before any is checked
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
                if (u < FC / 2) *reinterpret_cast<float2 *>(plane_elem(xlo, xhi, 2 * u)) = hv[k];
            }
            if (__syncthreads_or(!ok)) { aborted = true; break; }
        }
        stamp(l, 4, 0);
        wait_slot(0);
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            smem_rows_dot<1>(wreg4, 0, r < or1 ? 1 : 0, xlo, xhi, half * (CPR_D / 2), (half + 1) * (CPR_D / 2),
                             half * (CPR_D / 2), a);
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
        // drain this warp's bulk copies still in flight, then leave
        if (lane == 0)
            for (int i = 0; i < 2 + LM_NB; i++)
                if ((pend >> i) & 1u) mbar_wait(&mb[i], (phase >> i) & 1u);
        return;
    }
    // ================= LM head + argmax
    if (p.with_logits) {
        int v0, v1;
        share(V, b, G, v0, v1);
        // per warp: rows v0 + warp + 16j, LM_G at a time (one group: one
        // dot pass over x and LM_G independent reductions), through LM_NB
        // groups of row buffers in the head slot, each group filled by bulk
        // copies completing on its own mbarrier.  The first groups are
        // requested before the final norm's input arrives.
        const int nrow = max(0, (v1 - v0 - warp + WARPS - 1) / WARPS);
        const int ngrp = (nrow + LM_G - 1) / LM_G;
        auto issue_grp = [&](int k) {  // lane 0
            const int slot = k % LM_NB, j0 = k * LM_G, nj = min(LM_G, nrow - j0);
            issue_begin(2 + slot, (unsigned)nj * C * 2);
            for (int j = 0; j < nj; j++)
                bulk_g2s(wreg + (slot * LM_G + j) * C * 2, emb + (long)(v0 + warp + WARPS * (j0 + j)) * C, C * 2,
                         &mb[2 + slot]);
        };
        fence_async();
        if (lane == 0)
            for (int k = 0; k < min(LM_NB, ngrp); k++) issue_grp(k);
        const unsigned gwf = xact ? *reinterpret_cast<const unsigned *>(p.w + OFF_LNF / 2 + 2 * tid) : 0u;
        if (tid == 0) best_s = 0ull;
        if (!wait_x(epoch(NL - 1, 4))) {
            if (lane == 0)
                for (int i = 0; i < 2 + LM_NB; i++)
                    if ((pend >> i) & 1u) mbar_wait(&mb[i], (phase >> i) & 1u);
            return;
        }
        rms_regs(xv, gwf, xhw, xlw, red, eps);
        __syncthreads();
        unsigned long long best = 0ull;
        for (int k = 0; k < ngrp; k++) {
            const int slot = k % LM_NB, j0 = k * LM_G, nj = min(LM_G, nrow - j0);
            wait_slot(2 + slot);
            __syncwarp();
            float a[LM_G];
            smem_rows_dot_hl<LM_G>(wreg4 + slot * LM_G * CPR, CPR, nj, xh4, xl4, 0, CPR, 0, a);
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
        // CTA 0 finalises once every CTA's argmax is in
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
