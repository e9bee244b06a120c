// q8k.cuh -- the Q8_K activation quantizer for one 256-value block, one warp
// per block, 8 consecutive values per lane; shared by the quantize kernels
// (quantize.cu) and the matvec's fused quantize (matvec.cu), so that both
// produce the same bytes.  Restates quantize_row_q8_K_ref
// (src/kernels_quant.cpp:80-118); the rounding rules are listed at the top of
// quantize.cu.
#pragma once
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {

struct Q8KWarp {
    float d;        // stored fp32 scale (1/iscale, or 0 for an all-zero block)
    int8_t q[8];    // this lane's 8 quants
};

// The block's values 8*lane .. 8*lane+7 (coherent loads: an earlier kernel
// may have written them).
__device__ __forceinline__ void q8_K_load(const float* src, uint32_t lane, float (&v)[8])
{
    const float4 a = ld_dep_f4(src + lane * 8);
    const float4 b = ld_dep_f4(src + lane * 8 + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ Q8KWarp q8_K_warp_vals(const float (&v)[8], uint32_t lane)
{
    // the reference's strict '>' scan keeps the first element (in index
    // order) with the largest |x|: the largest |x| over the warp (NaNs never
    // win, as there), then the lowest lane holding it gives that element
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float vsel = 0.0f;
    bool hit = false;
#pragma unroll
    for (int j = 7; j >= 0; j--) {
        if (fabsf(v[j]) == amax) {
            vsel = v[j];
            hit = true;
        }
    }
    const uint32_t hits = __ballot_sync(0xffffffffu, hit);
    const float vmax = __shfl_sync(0xffffffffu, vsel, hits ? __ffs(hits) - 1 : 0);
    (void)lane;
    Q8KWarp r;
    if (amax == 0.0f) {
        r.d = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) r.q[j] = 0;
        return r;
    }
    const float iscale = __fdiv_rn(-127.0f, vmax);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float biased = __fmaf_rn(iscale, v[j], 12582912.0f);
        const int bits = __float_as_int(biased);
        const int q = (bits & 0x007fffff) - 0x00400000;
        r.q[j] = (int8_t)(q < 127 ? q : 127);
    }
    r.d = __fdiv_rn(1.0f, iscale);
    return r;
}

__device__ __forceinline__ Q8KWarp q8_K_warp(const float* src, uint32_t lane)
{
    float v[8];
    q8_K_load(src, lane, v);
    return q8_K_warp_vals(v, lane);
}

// This warp's block as a matvec record (kQ8KMvBytes at `out`, global or
// shared memory): quants of sub-block j (32 values), elements 8t..8t+7
// (t = 0..3), at byte 64*(j/2) + 16*t + 8*(j%2) -- lane 4j+t's eight bytes --
// so a lane's MMA B fragments of two sub-blocks are one 16-byte word and the
// four lanes of a fragment read 64 contiguous bytes; then the eight 32-element
// sums bsums[2j] + bsums[2j+1] as int16 at byte 256, and d (fp32) at byte 272.
__device__ __forceinline__ void q8_K_store_mv(uint8_t* out, const Q8KWarp& r, uint32_t lane)
{
    uint32_t lo = 0, hi = 0;
    int sum8 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) lo |= (uint32_t)(uint8_t)r.q[j] << (8 * j);
#pragma unroll
    for (int j = 0; j < 4; j++) hi |= (uint32_t)(uint8_t)r.q[4 + j] << (8 * j);
#pragma unroll
    for (int j = 0; j < 8; j++) sum8 += r.q[j];
    const uint32_t j = lane >> 2, t = lane & 3u;
    *reinterpret_cast<uint2*>(out + 64 * (j >> 1) + 16 * t + 8 * (j & 1u)) = make_uint2(lo, hi);
    int s32 = sum8 + __shfl_xor_sync(0xffffffffu, sum8, 1);
    s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
    if (t == 0) *reinterpret_cast<int16_t*>(out + kQKK + 2 * j) = (int16_t)s32;
    if (lane == 0) *reinterpret_cast<float*>(out + kQKK + 16) = r.d;
}

// Exact fp16 of a small integer (|q| < 512) without a conversion
// instruction: 1536 + q is an fp16 with unit spacing (bits 0x6600 + q), and
// subtracting 1536 from it is exact.
__device__ __forceinline__ __half small_int_half(int q)
{
    return __hsub(__ushort_as_half((unsigned short)(0x6600 + q)), __ushort_as_half((unsigned short)0x6600));
}
// The same for two values, (lo, hi) in one half2.
__device__ __forceinline__ __half2 small_int_half2(int lo, int hi)
{
    const uint32_t b = ((uint32_t)(0x6600 + lo) & 0xffffu) | ((uint32_t)(0x6600 + hi) << 16);
    const __half m = __ushort_as_half((unsigned short)0x6600);
    return __hsub2(*reinterpret_cast<const __half2*>(&b), __halves2half2(m, m));
}

// ---- Q8_0 (quantize_row_q8_0_ref, src/kernels_quant.cpp:120-144) ----

// roundf(x * id) -- half away from zero, after the rounded product -- as an
// integer, for |x * id| < 2^22 (the quantizer's products are at most 127 and
// a little), without conversion instructions: floor(|v| + 0.5) is roundf(|v|);
// adding 0.5 rounded toward zero keeps the floor of the exact sum, and adding
// 2^23 rounded toward zero leaves that floor in the low mantissa bits.  A NaN
// product gives 0, as the float -> int conversion does.
__device__ __forceinline__ int q8_0_round(float x, float id)
{
    const float v = __fmul_rn(x, id);
    const float t = __fadd_rz(__fadd_rz(fabsf(v), 0.5f), 8388608.0f);
    const int a = __float_as_int(t) - 0x4B000000;  // roundf(|v|); out of range for a NaN
    const int q = (unsigned)a < 256u ? a : 0;
    return v < 0.0f ? -q : q;
}

__device__ __forceinline__ int8_t q8_0_quant(float x, float id) { return static_cast<int8_t>(q8_0_round(x, id)); }

// Eight Q8_0 blocks (256 values) as one matvec record (kQ80MvBytes at
// `out`), one warp, the values 8*lane .. 8*lane+7 in v: block j = lane / 4
// is quantized by lanes 4j..4j+3 (d = amax/127 and 1/d as IEEE divisions,
// the stored fp16 scale round-to-nearest-even), its quants land where
// q8_K_store_mv puts sub-block j (byte 64*(j/2) + 16*t + 8*(j%2), t = lane %
// 4), and the stored scale, widened exactly to fp32, at byte 256 + 4*j.
__device__ __forceinline__ void q8_0_store_mv(uint8_t* out, const float (&v)[8], uint32_t lane)
{
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) lo |= (uint32_t)(uint8_t)q8_0_quant(v[k], id) << (8 * k);
#pragma unroll
    for (int k = 0; k < 4; k++) hi |= (uint32_t)(uint8_t)q8_0_quant(v[4 + k], id) << (8 * k);
    const uint32_t j = lane >> 2, t = lane & 3u;
    *reinterpret_cast<uint2*>(out + 64 * (j >> 1) + 16 * t + 8 * (j & 1u)) = make_uint2(lo, hi);
    if (t == 0) *reinterpret_cast<float*>(out + kQKK + 4 * j) = __half2float(__float2half_rn(d));
}

// This warp's block as a Q6_K matvec record (kQ8KQ6Bytes at `out`): d (fp32)
// at byte 0, the quants in their natural order at byte 16 (lane l's eight at
// 16 + 8l), the sixteen 16-element sums (int16) at byte 272.
__device__ __forceinline__ void q8_K_store_q6(uint8_t* out, const Q8KWarp& r, uint32_t lane)
{
    uint32_t lo = 0, hi = 0;
    int sum8 = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) lo |= (uint32_t)(uint8_t)r.q[j] << (8 * j);
#pragma unroll
    for (int j = 0; j < 4; j++) hi |= (uint32_t)(uint8_t)r.q[4 + j] << (8 * j);
#pragma unroll
    for (int j = 0; j < 8; j++) sum8 += r.q[j];
    *reinterpret_cast<uint2*>(out + 16 + 8 * lane) = make_uint2(lo, hi);
    const int s16 = sum8 + __shfl_xor_sync(0xffffffffu, sum8, 1);  // 16-element group = lane pair
    if ((lane & 1u) == 0) *reinterpret_cast<int16_t*>(out + 16 + kQKK + lane) = (int16_t)s16;
    if (lane == 0) *reinterpret_cast<float*>(out) = r.d;
}

}  // namespace pxq
