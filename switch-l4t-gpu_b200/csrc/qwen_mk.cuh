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
// Every input of a stage that does not depend on this step's activations
// (weights, norm gains, biases, RoPE cos/sin) is requested BEFORE the
// barrier that precedes the stage, so after it only the activations
// themselves cross L2 (one round trip).  Each CTA keeps its own residual
// rows on chip, so the residual adds need no re-read.
//
// Barrier waits are bounded: after SPIN_LIMIT polls the kernel sets *err,
// drains its own copies and returns; the host reports the error.
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
constexpr int WHEAD = 6 * C * 2;      // per-warp head slot: 6 rows of 896 fp16 (S1, S4, S5, LM head)
constexpr int WREG = WHEAD + C;       // + tail slot for the O half-row (896 B): 11648 B per warp
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

// ---- TMA bulk staging: one lane per warp issues cp.async.bulk (global ->
// shared, completing on an mbarrier) for whole row segments.  Bulk copies
// run on the TMA engine, so they do not queue in front of the ordinary
// loads (activations, barrier polls) of the stage that follows.
SB_DEV void mbar_init(uint64_t *mb, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mb)), "r"(count) : "memory");
}
SB_DEV void mbar_expect_tx(uint64_t *mb, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mb)), "r"(bytes) : "memory");
}
SB_DEV void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *mb) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(mb))
                 : "memory");
}
// Bounded wait for the mbarrier phase with parity `ph`; false on timeout.
SB_DEV bool mbar_wait(uint64_t *mb, unsigned ph) {
    for (long spin = 0; spin < (1L << 24); spin++) {
        unsigned done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(mb)), "r"(ph)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Copy `nchunks` 16-byte chunks of one weight row (starting at chunk c0)
// into shared memory, warp-cooperatively.
SB_DEV void warp_copy_row(void *dst, const unsigned short *row, int c0, int nchunks) {
    const int lane = threadIdx.x & 31;
    const uint4 *src = reinterpret_cast<const uint4 *>(row) + c0;
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int c = lane; c < nchunks; c += 32) cp_async16(d + c, src + c);
}

// Grid-wide barrier, split in two so a CTA can issue its prefetches for the
// coming stages in between (that time is spent waiting anyway).
// grid_arrive: all of this CTA's writes are ordered before a release
// increment of the counter.  grid_wait: returns false on timeout (after
// setting *err).  `target` = arrivals to wait for (k * gridDim.x at the k-th
// barrier).
// The arrive and the polling are done by POLLER, the first lane of the last
// warp: that warp issues its own prefetches only after the wait, so the
// poll starts as soon as the CTA has arrived.
constexpr int POLLER = THREADS - 32;
SB_DEV void grid_arrive(const Params &p, unsigned target) {
    __syncthreads();
    if (threadIdx.x == POLLER) {
        if (p.trace) {
            const unsigned idx = target / gridDim.x;  // 1-based barrier number
            if (idx < 128) p.trace[((size_t)blockIdx.x * 128 + idx) * 2] = globaltimer();
        }
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
    }
}
SB_DEV bool grid_wait(const Params &p, unsigned target, int *abort_s) {
    if (threadIdx.x == POLLER) {
        long spins = 0;
        while (ld_acquire(p.bar) < target) {
            if ((++spins & 255) == 0) {
                if (*(volatile int *)p.err) break;
                if (spins > SPIN_LIMIT) { atomicExch(p.err, 1); break; }
            }
        }
        *abort_s = *(volatile int *)p.err;
        if (p.trace) {
            const unsigned idx = target / gridDim.x;
            if (idx < 128) p.trace[((size_t)blockIdx.x * 128 + idx) * 2 + 1] = globaltimer();
        }
    }
    __syncthreads();
    return *abort_s == 0;
}
SB_DEV bool grid_sync(const Params &p, unsigned target, int *abort_s) {
    grid_arrive(p, target);
    return grid_wait(p, target, abort_s);
}

// Contiguous share [lo, hi) of n units for CTA b of g.
SB_DEV void share(int n, int b, int g, int &lo, int &hi) {
    lo = (int)((long)n * b / g);
    hi = (int)((long)n * (b + 1) / g);
}

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

// dot of one smem row (K/8 chunks) with the split x planes, lane-strided,
// chunk range [c0, c1) of the plane index.
SB_DEV float smem_row_dot(const uint4 *row, const float4 *lo, const float4 *hi, int c0, int c1, int row_c0) {
    float acc = 0.0f;
    for (int c = c0 + (threadIdx.x & 31); c < c1; c += 32) acc = dot_chunk(WH(), row[c - row_c0], lo[c], hi[c], acc);
    return acc;
}

// RMSNorm from registers: thread t < C/2 holds elements (2t, 2t+1) of x in
// xv and the two fp16 gains in gw (packed); writes x*inv*g into the split
// planes (element i lives in plane (i%8)<4 ? lo : hi, float (i/8)*4 + i%4).
SB_DEV void rms_regs(float2 xv, unsigned gw, float4 *lo, float4 *hi, float *red, float eps) {
    const int t = threadIdx.x;
    const bool act = t < C / 2;
    float s = act ? fmaf(xv.x, xv.x, xv.y * xv.y) : 0.0f;
    s = block_sum(s, red);
    const float inv = 1.0f / sqrtf(__fdiv_rn(s, (float)C) + eps);
    if (act) {
        const float g0 = h2f_ftz((unsigned short)(gw & 0xffffu)), g1 = h2f_ftz((unsigned short)(gw >> 16));
        const float2 y = make_float2(__fmul_rn(__fmul_rn(xv.x, inv), g0), __fmul_rn(__fmul_rn(xv.y, inv), g1));
        const int i = 2 * t, c = i / 8, j = i % 8;
        float *plane = reinterpret_cast<float *>(j < 4 ? lo : hi);
        *reinterpret_cast<float2 *>(plane + c * 4 + (j % 4)) = y;
    }
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
// dynamic smem: FC*4 + WARPS*WREG + score_cap*4 + (32 + WARPS*64 + WARPS)*4 bytes.
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
    float *opart = red + 32;            // WARPS x HD per-warp partial P.V
    float *ksum = opart + WARPS * HD;   // WARPS floats: split-K partials / per-warp softmax sums
    __shared__ int abort_s;
    __shared__ float wmax_s[WARPS], xown[8];
    __shared__ unsigned long long best_s;
    __shared__ __align__(8) uint64_t mbar[WARPS][2 + LM_NB];

    const int b = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    unsigned char *wreg = wbase + (size_t)warp * WREG;
    const uint4 *wreg4 = reinterpret_cast<const uint4 *>(wreg);
    unsigned target = 0;
    if (tid == 0) abort_s = 0;
    if (sb_step_idle(p.st)) return;  // uniform: every CTA reads the same state
    if (lane == 0)
        for (int i = 0; i < 2 + LM_NB; i++) mbar_init(&mbar[warp][i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    if (p.trace && tid == 0) p.trace[(size_t)b * 256] = globaltimer();  // slot 0: start
    const int pos = p.st->pos, T = pos + 1;
    const int tok = p.tokens[pos];
    const float eps = 1e-6f;
    const unsigned short *emb = p.w;
    const float *cosT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_COS);
    const float *sinT = reinterpret_cast<const float *>(reinterpret_cast<const char *>(p.w) + OFF_SIN);
    const bool xact = tid < C / 2;  // holds x elements (2 tid, 2 tid + 1) in RMS stages

    // per-CTA shares (static over the step)
    int qp0, qp1, or0, or1, gp0, gp1;
    share(QKV / 2, b, G, qp0, qp1);  // RoPE pairs
    share(C, b, G, or0, or1);        // O rows and down rows (this CTA's residual rows)
    share(FC, b, G, gp0, gp1);       // gate/up pairs
    // attention T-splits: ~48 positions per item (a warp holds up to 4
    // positions' K/V in registers), at most p.splits per head
    const int nsplit = max(1, min(p.splits, (T + 47) / 48));
    const int slen = (T + nsplit - 1) / nsplit;

    auto layer_ptr = [&](int l) { return p.w + (LBASE / 2) + (long)l * (LSTRIDE / 2); };

    // L2 prefetch of this CTA's slices of layer l, in five pieces of ~40 KB
    // (one per stage) so the weight stream is spread evenly over the layer
    // instead of bursting in front of the latency-critical barrier and
    // activation traffic.  Issued by one lane (not the barrier poller).
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
    // [2 + k]: LM-head ring slot k.  `phase` bit i = parity to wait for next.
    unsigned phase = 0;
    uint64_t *mb = mbar[warp];
    auto issue_begin = [&](int i, unsigned bytes) {  // lane 0 only
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier generic reads of the slot
        mbar_expect_tx(&mb[i], bytes);
    };
    auto wait_slot = [&](int i) {
        if (!mbar_wait(&mb[i], (phase >> i) & 1u) && lane == 0) atomicExch(p.err, 2);
        phase ^= 1u << i;
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
    // gate/up pairs gp0 + warp + 16k, k < 3, rows (gate_k, up_k): the byte
    // count of all pairs is announced with the first piece, then one pair is
    // issued per stage (S1 arrive, S2, S3) to spread the traffic
    auto copy_s4_piece = [&](int l, int k) {
        if (lane != 0) return;
        const int npair = min(3, max(0, (gp1 - (gp0 + warp) + WARPS - 1) / WARPS));
        if (k == 0) issue_begin(0, (unsigned)npair * 2 * C * 2);
        if (k < npair) {
            const unsigned short *W = layer_ptr(l) + L_GATEUP;
            const int i = gp0 + warp + WARPS * k;
            bulk_g2s(wreg + (2 * k) * C * 2, W + (long)i * C, C * 2, &mb[0]);
            bulk_g2s(wreg + (2 * k + 1) * C * 2, W + (long)(FC + i) * C, C * 2, &mb[0]);
        }
    };
    auto copy_s5 = [&](int l) {  // down rows: warp w -> row or0 + w/2, half w%2 of K
        if (lane != 0) return;
        const int r = or0 + warp / 2, half = warp % 2;
        issue_begin(0, r < or1 ? FC : 0);
        if (r < or1) bulk_g2s(wreg, layer_ptr(l) + L_DOWN + (long)r * FC + half * (FC / 2), FC, &mb[0]);
    };
    // Split-K (2 warps per row) reduction + residual update of this CTA's rows.
    auto resid_update = [&](float a) {
        if (lane == 0) ksum[warp] = a;
        __syncthreads();
        if (tid < or1 - or0) {
            const float y = ksum[2 * tid] + ksum[2 * tid + 1];
            const float xn = __fadd_rn(xown[tid], y);
            xown[tid] = xn;
            p.x[or0 + tid] = xn;
        }
    };

    // ---- prologue: this CTA's residual rows start as the embedding
    if (tid < or1 - or0) xown[tid] = h2f_ftz(emb[(long)tok * C + or0 + tid]);
    if (prefetcher)
        for (int piece = 0; piece < 5; piece++) prefetch_piece(0, piece);
    copy_s1(0);
    // layer-0 S1 input: the embedding row (constant: no barrier needed)
    float2 xv = make_float2(0.f, 0.f);
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
    bool pending_s1 = false;

    for (int l = 0; l < NL; l++) {
        const unsigned short *L = layer_ptr(l);
        float *kc = p.kv + (long)l * p.ctx_cap * KVD;
        float *vc = p.kv + (long)(NL + l) * p.ctx_cap * KVD;
        // ================= S1: RMSNorm -> QKV -> RoPE -> q / cache
        if (l > 0) {
            if (!grid_wait(p, target, &abort_s)) break;  // arrival was at the end of S5
            if (pending_s1) {  // the poller's warp: its S1 copies and constants now
                copy_s1(l);
                s1_consts(l);
                pending_s1 = false;
            }
            if (xact) xv = __ldcg(reinterpret_cast<const float2 *>(p.x) + tid);
        }
        rms_regs(xv, gw1, xlo, xhi, red, eps);
        __syncthreads();
        if (prefetcher) {
            prefetch_piece(l + 1, 0);
            if (p.with_logits && l >= NL - 4) {  // first ~512 KB of this CTA's LM-head rows
                int v0, v1;
                share(V, b, G, v0, v1);
                const long r0 = v0 + (long)(l - (NL - 4)) * 73, r1 = min((long)v1, r0 + 73);
                prefetch_rows(emb, C * 2, r0, r1, 1L << 20);
            }
        }
        wait_slot(0);
        __syncwarp();
        if (pp1 < qp1) {
            const int h = pp1 / 32, i = pp1 % 32;
            const int r0 = h * HD + i, r1 = r0 + 32;
            float a[2];
            smem_rows_dot<2>(wreg4, CPR, 2, xlo, xhi, 0, CPR, 0, a);
            const float a0 = warp_sum(a[0]), a1 = warp_sum(a[1]);
            if (lane == 0) {
                float y0 = __fadd_rn(a0, b0), y1 = __fadd_rn(a1, b1);
                if (h < NH + NKV) {
                    const float o0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                    const float o1 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs));
                    y0 = o0;
                    y1 = o1;
                }
                if (h < NH) { p.q[r0] = y0; p.q[r1] = y1; }
                else if (h < NH + NKV) { kc[(long)pos * KVD + r0 - C] = y0; kc[(long)pos * KVD + r1 - C] = y1; }
                else { vc[(long)pos * KVD + r0 - C - KVD] = y0; vc[(long)pos * KVD + r1 - C - KVD] = y1; }
            }
        }
        target += G;
        grid_arrive(p, target);
        // O rows (tail slot) and gate/up rows (head slot; S1's rows are
        // consumed) arrive while the barriers, attention and O run; the
        // poller's warp issues its copies after the wait
        if (warp != WARPS - 1) { copy_s3(l); copy_s4_piece(l, 0); }
        // ================= S2: attention partials; a warp per position, K and V
        // rows loaded together so one L2 round trip serves scores and P.V
        if (!grid_wait(p, target, &abort_s)) break;
        if (warp == WARPS - 1) { copy_s3(l); copy_s4_piece(l, 0); }
        copy_s4_piece(l, 1);
        if (prefetcher) prefetch_piece(l + 1, 1);
        for (int item = b; item < NH * nsplit; item += G) {
            const int h = item / nsplit, s = item % nsplit, g = h / (NH / NKV);
            const int t0 = s * slen, t1 = min(T, t0 + slen), n = max(0, t1 - t0);
            const float2 q2 = __ldcg(reinterpret_cast<const float2 *>(p.q + h * HD) + lane);
            // each warp keeps up to 4 positions' scores and V rows in registers
            float sc[4];
            float2 vv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int j = warp + WARPS * k;
                sc[k] = -1e30f;
                vv[k] = make_float2(0.f, 0.f);
                if (j < n) {
                    const float2 k2 = __ldcg(reinterpret_cast<const float2 *>(kc + (long)(t0 + j) * KVD + g * HD) + lane);
                    vv[k] = __ldcg(reinterpret_cast<const float2 *>(vc + (long)(t0 + j) * KVD + g * HD) + lane);
                    sc[k] = warp_sum(fmaf(q2.x, k2.x, q2.y * k2.y)) * 0.125f;
                }
            }
            // positions beyond 64 per item (long contexts): scores via smem, V re-read
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) {
                const float2 k2 = __ldcg(reinterpret_cast<const float2 *>(kc + (long)(t0 + j) * KVD + g * HD) + lane);
                const float d = warp_sum(fmaf(q2.x, k2.x, q2.y * k2.y)) * 0.125f;
                if (lane == 0) scores[j] = d;
            }
            __syncwarp();
            float wm = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
            for (int j = warp + 4 * WARPS; j < n; j += WARPS) wm = fmaxf(wm, scores[j]);
            if (lane == 0) wmax_s[warp] = wm;
            __syncthreads();
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
                const float e = expf(scores[j] - m);
                lsum += e;
                const float2 v2 = __ldcg(reinterpret_cast<const float2 *>(vc + (long)(t0 + j) * KVD + g * HD) + lane);
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
                float *pp = p.part + (long)(h * p.splits + s) * (HD + 2);
                pp[tid] = acc;
                if (tid == 0) {
                    float ls = 0.f;
#pragma unroll
                    for (int w = 0; w < WARPS; w++) ls += ksum[w];
                    pp[HD] = m;
                    pp[HD + 1] = ls;
                }
            }
            __syncthreads();
        }
        target += G;
        grid_arrive(p, target);
        // ================= S3: combine partials -> att; O rows; x += O att
        if (!grid_wait(p, target, &abort_s)) break;
        copy_s4_piece(l, 2);
        if (prefetcher) prefetch_piece(l + 1, 2);
        // 28 (head, 32-dim half) tasks over 16 warps (two per warp at most);
        // every partial a lane needs for both tasks is requested in one batch
        {
            float mv[2], lv[2], ov[2][16];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int task = warp + WARPS * u;
                const int h = task >> 1, d = (task & 1) * 32 + lane;
                const bool live = task < 2 * NH;
                const float *base = p.part + (long)(h * p.splits) * (HD + 2);
                mv[u] = -1e30f;
                lv[u] = 0.f;
                if (live && lane < nsplit) {
                    mv[u] = __ldcg(base + (long)lane * (HD + 2) + HD);
                    lv[u] = __ldcg(base + (long)lane * (HD + 2) + HD + 1);
                }
#pragma unroll
                for (int s2 = 0; s2 < 16; s2++) ov[u][s2] = (live && s2 < nsplit) ? __ldcg(base + (long)s2 * (HD + 2) + d) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int task = warp + WARPS * u;
                if (task >= 2 * NH) break;
                const int h = task >> 1, d = (task & 1) * 32 + lane;
                const float M = warp_max(mv[u]);
                const float wgt = (lane < nsplit) ? expf(mv[u] - M) : 0.f;
                const float Lsum = warp_sum(wgt * lv[u]);
                float acc = 0.f;
#pragma unroll
                for (int s2 = 0; s2 < 16; s2++) acc = fmaf(__shfl_sync(SB_FULL, wgt, s2), ov[u][s2], acc);
                const int c = d / 8, j = d % 8;
                reinterpret_cast<float *>(j < 4 ? xlo : xhi)[(h * HD / 8 + c) * 4 + (j % 4)] = acc / Lsum;
            }
        }
        __syncthreads();
        wait_slot(1);  // the O half-row (the gate/up rows may still be landing)
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            smem_rows_dot<1>(wreg4 + WHEAD / 16, 0, r < or1 ? 1 : 0, xlo, xhi, half * (CPR / 2), (half + 1) * (CPR / 2),
                             half * (CPR / 2), a);
            resid_update(warp_sum(a[0]));
        }
        target += G;
        grid_arrive(p, target);
        const unsigned gw4 = xact ? *reinterpret_cast<const unsigned *>(L + L_POST + 2 * tid) : 0u;
        // ================= S4: RMSNorm -> gate/up -> SwiGLU -> hid
        if (!grid_wait(p, target, &abort_s)) break;
        if (prefetcher) prefetch_piece(l + 1, 3);
        if (xact) xv = __ldcg(reinterpret_cast<const float2 *>(p.x) + tid);
        rms_regs(xv, gw4, xlo, xhi, red, eps);
        __syncthreads();
        wait_slot(0);
        __syncwarp();
        {
            // this warp's pairs: gp0 + warp + 16k, k < 3; rows stored (gate_k, up_k)
            const int npair = min(3, max(0, (gp1 - (gp0 + warp) + WARPS - 1) / WARPS));
            float a[6];
            smem_rows_dot<6>(wreg4, CPR, 2 * npair, xlo, xhi, 0, CPR, 0, a);
#pragma unroll
            for (int k = 0; k < 3; k++) {
                const float ag = warp_sum(a[2 * k]), au = warp_sum(a[2 * k + 1]);
                if (k < npair && lane == 0)
                    p.hid[gp0 + warp + WARPS * k] = __fmul_rn(__fdiv_rn(ag, __fadd_rn(1.0f, expf(-ag))), au);
            }
        }
        target += G;
        grid_arrive(p, target);
        if (warp != WARPS - 1) copy_s5(l);
        // ================= S5: down rows (split-K over warp pairs); x += down hid
        if (!grid_wait(p, target, &abort_s)) break;
        if (warp == WARPS - 1) copy_s5(l);
        if (prefetcher) prefetch_piece(l + 1, 4);
        for (int c = tid; c < CPR_D; c += blockDim.x) {
            xlo[c] = __ldcg(reinterpret_cast<const float4 *>(p.hid) + 2 * c);
            xhi[c] = __ldcg(reinterpret_cast<const float4 *>(p.hid) + 2 * c + 1);
        }
        __syncthreads();
        wait_slot(0);
        __syncwarp();
        {
            const int r = or0 + warp / 2, half = warp % 2;
            float a[1];
            smem_rows_dot<1>(wreg4, 0, r < or1 ? 1 : 0, xlo, xhi, half * (CPR_D / 2), (half + 1) * (CPR_D / 2),
                             half * (CPR_D / 2), a);
            resid_update(warp_sum(a[0]));
        }
        target += G;
        grid_arrive(p, target);  // waited at the top of the next layer (or before the LM head)
        if (l + 1 < NL && warp != WARPS - 1) {
            copy_s1(l + 1);
            s1_consts(l + 1);
        }
        if (l + 1 < NL && warp == WARPS - 1) {  // after the poll: the wait at the top of S1
            pending_s1 = true;
        }
    }
    if (abort_s) return;
    // ================= LM head + argmax
    const unsigned gwf = xact ? *reinterpret_cast<const unsigned *>(p.w + OFF_LNF / 2 + 2 * tid) : 0u;
    if (!grid_wait(p, target, &abort_s)) return;
    if (p.with_logits) {
        if (xact) xv = __ldcg(reinterpret_cast<const float2 *>(p.x) + tid);
        if (tid == 0) best_s = 0ull;
        rms_regs(xv, gwf, xlo, xhi, red, eps);
        __syncthreads();
        int v0, v1;
        share(V, b, G, v0, v1);
        // per warp: rows v0 + warp + 16k through a ring of LM_NB row buffers,
        // each filled by a bulk copy completing on its own mbarrier
        unsigned long long best = 0ull;
        for (int k = 0; k < LM_NB; k++) {
            const int r = v0 + warp + WARPS * k;
            if (r < v1 && lane == 0) {
                issue_begin(2 + k, C * 2);
                bulk_g2s(wreg + k * C * 2, emb + (long)r * C, C * 2, &mb[2 + k]);
            }
        }
        for (int k = 0;; k++) {
            const int r = v0 + warp + WARPS * k;
            if (r >= v1) break;
            const int slot = k % LM_NB;
            wait_slot(2 + slot);
            __syncwarp();
            float a[1];
            smem_rows_dot<1>(wreg4 + slot * CPR, 0, 1, xlo, xhi, 0, CPR, 0, a);
            const float dotv = warp_sum(a[0]);
            if (lane == 0) p.logits[r] = dotv;
            const unsigned long long key = argmax_key(dotv, r);
            best = key > best ? key : best;
            __syncwarp();
            const int rn = v0 + warp + WARPS * (k + LM_NB);
            if (rn < v1 && lane == 0) {
                issue_begin(2 + slot, C * 2);
                bulk_g2s(wreg + slot * C * 2, emb + (long)rn * C, C * 2, &mb[2 + slot]);
            }
        }
        if (lane == 0 && best) atomicMax(&best_s, best);
        __syncthreads();
        if (tid == 0 && best_s) atomicMax(&p.st->key, best_s);
        target += G;
        if (!grid_sync(p, target, &abort_s)) return;
    }
    // ================= finalize (one thread of CTA 0), as sb_finalize
    if (b == 0 && tid == 0) {
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
