// sb_mk_common.cuh -- pieces shared by the persistent whole-step decode
// kernels (qwen_decode_mk, gpt2_decode_mk): the parameter view, flagged
// exchange words, bounded waits, mbarriers, TMA bulk copies and the
// contiguous share of a range per CTA.
//
// Flagged words: an activation value is stored as one 8-byte word
// (float bits | epoch << 32) with a single relaxed 64-bit store; a consumer
// polls the words it needs until their epoch is the current one.  A 64-bit
// aligned access is single-copy atomic, so a word whose epoch matches
// carries its value -- no fence and no counter between stages.
#pragma once
#include "sb_common.cuh"
#include "sb_mk_params.h"
#include "sb_step.h"

namespace mkc {

typedef unsigned long long u64;
constexpr long LL_SPIN_LIMIT = 1L << 21;  // polls (~a second) before giving up

// Typed view of SbMkParams.
struct Params {
    const unsigned short *w; // weight file image
    float *kv;               // [2][NL][ctx][KVD]
    u64 *ll;                 // flagged words
    float *logits;           // [V]
    SbStep *st;
    int *tokens;
    unsigned *sync;          // [0] step sequence number, [1] LM-head arrivals
    int *err;                // set on a wait timeout
    unsigned long long *trace;
    int ctx_cap;
    int with_logits;
    int splits;              // attention T-splits per head (<= SPLITS_MAX)
    int score_cap;           // positions per split the score buffer holds
    int test_stall;          // test hook (SbMkParams.test_stall)
    SB_DEV explicit Params(const SbMkParams &r)
        : w((const unsigned short *)r.w), kv((float *)r.kv), ll((u64 *)r.ll), logits((float *)r.logits),
          st((SbStep *)r.st), tokens((int *)r.tokens), sync((unsigned *)r.sync), err((int *)r.err),
          trace((unsigned long long *)r.trace), ctx_cap(r.ctx_cap), with_logits(r.with_logits),
          splits(r.splits), score_cap(r.score_cap), test_stall(r.test_stall) {}
};

// ------------------------------------------------------------------ PTX helpers
SB_DEV unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
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

// ---- flagged words
SB_DEV u64 ll_word(float v, unsigned e) { return ((u64)e << 32) | __float_as_uint(v); }
SB_DEV void ll_put(u64 *p, float v, unsigned e) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(ll_word(v, e)) : "memory");
}
SB_DEV u64 ll_get(const u64 *p) {
    u64 v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
SB_DEV void ll_get2(const u64 *p, u64 &a, u64 &b) {
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
SB_DEV bool ll_is(u64 w, unsigned e) { return (unsigned)(w >> 32) == e; }
SB_DEV float ll_val(u64 w) { return __uint_as_float((unsigned)w); }
// Called after a poll found stale words: every 64 polls stop if another CTA
// gave up, or give up after the limit.  (A back-off sleep between polls was
// measured slower: the added detection delay outweighs the L2 traffic saved.)
SB_DEV bool ll_keep_polling(long spin, int *err) {
    if ((spin & 63) != 63) return true;
    if (*(volatile int *)err) return false;
    if (spin > LL_SPIN_LIMIT) {
        atomicExch(err, 3);
        return false;
    }
    return true;
}
// The pair of words at p (16-byte aligned) once both carry epoch e.
SB_DEV bool ll_wait2(const u64 *p, unsigned e, float &a, float &b, int *err) {
    for (long spin = 0;; spin++) {
        u64 w0, w1;
        ll_get2(p, w0, w1);
        if (ll_is(w0, e) && ll_is(w1, e)) {
            a = ll_val(w0);
            b = ll_val(w1);
            return true;
        }
        if (!ll_keep_polling(spin, err)) return false;
    }
}

// ---- TMA bulk staging: one lane per warp issues cp.async.bulk (global ->
// shared, completing on an mbarrier) for whole row segments.  Bulk copies
// run on the TMA engine, so they do not queue in front of the ordinary
// loads (activation words, polls) of the stage that follows.
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

// Block-wide sum for the step kernels with one barrier: the warp partials go
// to red[off .. off + 16), and the caller alternates `off` (0 / 16) between
// consecutive reductions, so a reduction never overwrites partials another
// warp may still be reading (the stage code between two uses of the same
// half always passes a barrier).  THREADS = 512 (16 warps).
SB_DEV float block_sum1(float v, float *red, int off) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0) red[off + w] = v;
    __syncthreads();
    float s = (lane < 16) ? red[off + lane] : 0.0f;
    return warp_sum(s);
}

// Contiguous share [lo, hi) of n units for CTA b of g.
SB_DEV void share(int n, int b, int g, int &lo, int &hi) {
    lo = (int)((long)n * b / g);
    hi = (int)((long)n * (b + 1) / g);
}

}  // namespace mkc
