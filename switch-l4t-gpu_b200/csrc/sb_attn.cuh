// sb_attn.cuh -- split-T decode attention ("flash-decode") over an FP32 KV
// cache, shared by the Qwen (GQA, 7 query heads per KV head) and GPT-2 (MHA)
// modules.
//
// One CTA per (KV group g, time split s).  A CTA scores its positions for
// the G query heads of group g, takes a split-local softmax (max m, sum l),
// and accumulates sum_t p_t v_t.  Partials (o, m, l) go to a scratch buffer;
// the last CTA of each group (atomic ticket) rescales them by exp(m_s - M)
// and writes out = sum_s e^(m_s-M) o_s / sum_s e^(m_s-M) l_s.  That equals
// the reference softmax-then-mix (qwen_engine.c:324-342, gpt2_engine.c:379-397)
// up to float rounding, but spreads T over many SMs instead of the
// reference's one thread per head looping serially over T
// (qwen_kernels.cu:147-164).
//
// The number of live splits is derived on the device from T = *pos + 1, so
// one launch shape (grid.y = max_splits) serves every decode position and can
// be captured in a CUDA graph.  CTAs beyond the live split count exit.
#pragma once
#include "sb_common.cuh"

#define SB_ATTN_HD 64
#define SB_ATTN_THREADS 128
#define SB_ATTN_MAXLEN 64  // positions per split at most

// per (group, split): G heads x (HD + 2) floats: o[0..63], m, l
template <int G>
__device__ void attn_decode_body(const float *__restrict__ q, const float *__restrict__ kc,
                                 const float *__restrict__ vc, int T, float *__restrict__ out,
                                 float *__restrict__ part, unsigned *__restrict__ counters,
                                 int kv_stride, float scale, int max_splits) {
    constexpr int HD = SB_ATTN_HD;
    __shared__ float q_s[G][HD];
    __shared__ float p_s[G][SB_ATTN_MAXLEN];
    __shared__ float m_s[G], l_s[G];
    __shared__ int last_s;

    const int g = blockIdx.x, s = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    // live split count and split length for this T
    int nsplit = (T + 15) / 16;
    if (nsplit > max_splits) nsplit = max_splits;
    int slen = (T + nsplit - 1) / nsplit;
    if (slen > SB_ATTN_MAXLEN) {  // host sizes max_splits so this cannot happen
        slen = SB_ATTN_MAXLEN;
    }
    if (s >= nsplit) return;
    const int t0 = s * slen;
    int t1 = t0 + slen;
    if (t1 > T) t1 = T;
    const int n = t1 - t0;

    for (int i = tid; i < G * HD; i += blockDim.x) q_s[i / HD][i % HD] = q[(g * G + i / HD) * HD + i % HD];
    __syncthreads();

    // scores: one warp per position, lanes own dims (2*lane, 2*lane+1)
    for (int j = warp; j < n; j += nwarps) {
        const float2 k2 = *reinterpret_cast<const float2 *>(kc + (size_t)(t0 + j) * kv_stride + g * HD + 2 * lane);
#pragma unroll
        for (int h = 0; h < G; h++) {
            float d = fmaf(q_s[h][2 * lane], k2.x, q_s[h][2 * lane + 1] * k2.y);
            d = warp_sum(d);
            if (lane == 0) p_s[h][j] = d * scale;
        }
    }
    __syncthreads();
    // split-local softmax numerators
    for (int h = warp; h < G; h += nwarps) {
        float m = -1e30f;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, p_s[h][j]);
        m = warp_max(m);
        float l = 0.0f;
        for (int j = lane; j < n; j += 32) {
            float e = expf(p_s[h][j] - m);
            p_s[h][j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { m_s[h] = m; l_s[h] = l; }
    }
    __syncthreads();
    // o[h][d] = sum_j p[h][j] v[t0+j][g*HD + d]
    for (int i = tid; i < G * HD; i += blockDim.x) {
        const int h = i / HD, d = i % HD;
        float acc = 0.0f;
        for (int j = 0; j < n; j++) acc = fmaf(p_s[h][j], vc[(size_t)(t0 + j) * kv_stride + g * HD + d], acc);
        float *pp = part + ((size_t)(g * max_splits + s) * G + h) * (HD + 2);
        pp[d] = acc;
        if (d == 0) { pp[HD] = m_s[h]; pp[HD + 1] = l_s[h]; }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned prev = atomicAdd(&counters[g], 1u);
        last_s = (prev == (unsigned)nsplit - 1u);
    }
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    for (int i = tid; i < G * HD; i += blockDim.x) {
        const int h = i / HD, d = i % HD;
        float M = -1e30f;
        for (int k = 0; k < nsplit; k++)
            M = fmaxf(M, __ldcg(part + ((size_t)(g * max_splits + k) * G + h) * (HD + 2) + HD));
        float L = 0.0f, o = 0.0f;
        for (int k = 0; k < nsplit; k++) {
            const float *pp = part + ((size_t)(g * max_splits + k) * G + h) * (HD + 2);
            float w = expf(__ldcg(pp + HD) - M);
            L = fmaf(w, __ldcg(pp + HD + 1), L);
            o = fmaf(w, __ldcg(pp + d), o);
        }
        out[(g * G + h) * HD + d] = o / L;
    }
    if (tid == 0) counters[g] = 0u;  // ready for the next launch
}
