// sb_common.cuh -- device helpers shared by every sm_100a module of this
// package: fp16 decode with the reference's flush-to-zero rule, streaming
// loads, warp/block reductions, programmatic-dependent-launch controls and
// L2 bulk prefetch.
#pragma once
#include <stdint.h>
#include <cuda_fp16.h>

#define SB_DEV __device__ __forceinline__
#define SB_FULL 0xffffffffu

// ---------------------------------------------------------------- fp16 decode
// The reference decodes weights with exponent-0 values flushed to +-0 and no
// inf/NaN handling (qwen_kernels.cu:6-14, qwen_engine.c:90-98).  For every
// normal fp16 value that is exactly the IEEE conversion, so we clear the
// subnormal halves of a packed pair and use the hardware conversion.
SB_DEV uint32_t ftz_half2_bits(uint32_t w) {
    // per 16-bit half: exponent field nonzero -> keep, else clear the half
    uint32_t e = w & 0x7C007C00u;
    uint32_t t = ((e + 0x7FFF7FFFu) & 0x80008000u) >> 15;  // bit0 / bit16 set if exp != 0
    return w & (t * 0xFFFFu);
}
SB_DEV float2 h2x2_ftz(uint32_t w) {
    uint32_t k = ftz_half2_bits(w);
    __half2 h = *reinterpret_cast<__half2 *>(&k);
    return __half22float2(h);
}
SB_DEV float h2f_ftz(uint16_t h) {
    return ((h & 0x7C00u) == 0) ? 0.0f : __half2float(__ushort_as_half(h));
}

// ---------------------------------------------------------------- packed FP32
// Blackwell's two-wide FP32 FMA (fma.rn.f32x2): halves the FMA instruction
// count of the dot products; each lane is still an IEEE FP32 fused
// multiply-add.
SB_DEV unsigned long long f2_pack(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
SB_DEV float f2_sum(unsigned long long v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return a + b;
}
SB_DEV void f2_unpack(unsigned long long v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
SB_DEV unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// acc += 8 fp16 weights (no subnormal flush: the data is pre-flushed) x 8 floats.
SB_DEV unsigned long long dot8_h_f2(const uint4 &w, const float4 &lo, const float4 &hi, unsigned long long acc) {
    const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
    const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
    const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&w.z));
    const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&w.w));
    acc = ffma2(f2_pack(f0.x, f0.y), f2_pack(lo.x, lo.y), acc);
    acc = ffma2(f2_pack(f1.x, f1.y), f2_pack(lo.z, lo.w), acc);
    acc = ffma2(f2_pack(f2.x, f2.y), f2_pack(hi.x, hi.y), acc);
    acc = ffma2(f2_pack(f3.x, f3.y), f2_pack(hi.z, hi.w), acc);
    return acc;
}

// ---------------------------------------------------------------- loads
// Weights are read exactly once per decode step: no L1 allocation, and a
// 256-byte L2 fetch granule so DRAM sees full bursts.
SB_DEV uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
SB_DEV float4 ld_f4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }

// Issue a bulk L2 prefetch of [p, p+bytes).  p and bytes must be 16-byte
// multiples; the copy engine splits it, nothing is written to shared memory.
SB_DEV void l2_prefetch_bulk(const void *p, uint32_t bytes) {
    if (bytes == 0) return;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialisation attribute may start while its predecessor drains.
// Everything before pdl_wait() must not read the predecessor's outputs.
SB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- reductions
SB_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(SB_FULL, v, o);
    return v;
}
SB_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(SB_FULL, v, o));
    return v;
}
// Block-wide sum; every thread gets the result.  `red` holds >= 32 floats.
SB_DEV float block_sum(float v, float *red) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float s = (lane < nw) ? red[lane] : 0.0f;
    s = warp_sum(s);
    return s;
}

// Order-preserving map float -> uint32 (larger float -> larger key).
SB_DEV uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// 64-bit argmax key: value key in the high word, complemented index in the
// low word, so atomicMax picks the largest value and, on ties, the FIRST
// index -- the reference's strict '>' scan (qwen_engine.c:360-364).
SB_DEV unsigned long long argmax_key(float v, int idx) {
    return ((unsigned long long)float_key(v) << 32) | (uint32_t)(~(uint32_t)idx);
}
SB_DEV int argmax_key_index(unsigned long long k) { return (int)(~(uint32_t)(k & 0xffffffffu)); }
