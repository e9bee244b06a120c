// matvec.cu -- small-M (decode) quantized matvec: y = X * W^T for M <= 8.
//
// Restates, for columns <= 8, the inner loop of cpu_quant_matmul
// (src/kernels_quant.cpp:389-400) with the dots pix_dot_q8_0 (:339-365) and
// pix_dot_q5_K (:163-254) on GPU: activations are the reference's Q8_0 /
// Q8_K blocks (produced by quantize.cu), weights stream straight from the raw
// GGUF rows in HBM.
//
// Mapping.  A CTA of 4 warps owns 16 weight rows; its warps split the K
// blocks round-robin.  Each K block (32 values) is one int8 tensor-core
// mma.sync m16n8k32: A = the 16 weight rows (unpacked in registers), B = the
// up-to-8 activation rows (n = activation row, zero-padded).  The exact int32
// block dot comes out of the MMA; the per-block fp32 scaling and the Q5_K
// sub-block scales / min term are applied in registers exactly as the
// reference does (int32 super-block sums, then one fp32 FMA per super-block).
// The K order inside a 32-block is permuted identically for A and B (legal:
// a dot product does not depend on the order of its terms) so that each
// thread's 8 weight bytes per block are contiguous in memory.
// Partial sums of the 4 warps are combined in shared memory in fixed order,
// so results are deterministic.
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int kRowsPerCta = 16;
constexpr int kWarps = 4;

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// 8 bytes from a 2-byte-aligned global address (Q8_0 blocks are 34 bytes).
__device__ __forceinline__ uint2 ld8_unaligned(const uint8_t* p)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    const uint32_t w0 = __ldg(w), w1 = __ldg(w + 1);
    const uint32_t w2 = sh ? __ldg(w + 2) : 0u;  // only touch the third word when the span needs it
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

__device__ __forceinline__ float ld_half(const uint8_t* p)
{
    return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(p))));
}

// ---------------------------------------------------------------- Q8_0 ------

__global__ void __launch_bounds__(128) k_matvec_q8_0(const uint8_t* __restrict__ w, int64_t stride, int64_t rows,
                                                     int64_t inner, const uint8_t* __restrict__ xq, int64_t columns,
                                                     float* __restrict__ y, int64_t ldy, const float* __restrict__ bias)
{
    __shared__ float part[kWarps][kRowsPerCta][8];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const int64_t r0 = (int64_t)blockIdx.x * kRowsPerCta;
    const int64_t ra = r0 + g, rb = r0 + g + 8;
    const bool va = ra < rows, vb = rb < rows;
    const int64_t nb = inner / kQK8_0;
    const int64_t xstride = nb * kQ8_0Bytes;
    const bool vx = (int64_t)g < columns;  // B column n = g is activation row g
    const uint8_t* wa = w + (va ? ra : 0) * stride;
    const uint8_t* wb = w + (vb ? rb : 0) * stride;
    const uint8_t* xr = xq + (vx ? g : 0) * xstride;
    // this thread's two output columns (activation rows) are 2t and 2t+1
    const uint8_t* xc0 = xq + min((int64_t)(2 * t), columns - 1) * xstride;
    const uint8_t* xc1 = xq + min((int64_t)(2 * t + 1), columns - 1) * xstride;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t b = warp; b < nb; b += kWarps) {
        const int64_t off = b * kQ8_0Bytes;
        uint2 qa = va ? ld8_unaligned(wa + off + 2 + 8 * t) : make_uint2(0, 0);
        uint2 qb = vb ? ld8_unaligned(wb + off + 2 + 8 * t) : make_uint2(0, 0);
        uint2 qx = vx ? ld8_unaligned(xr + off + 2 + 8 * t) : make_uint2(0, 0);
        const uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
        int d[4];
        mma_s8(d, a, qx.x, qx.y);
        const float dwa = va ? ld_half(wa + off) : 0.f, dwb = vb ? ld_half(wb + off) : 0.f;
        const float dx0 = ld_half(xc0 + off), dx1 = ld_half(xc1 + off);
        // pix_dot_q8_0: acc = fma(fp16(dw) * fp16(dx), float(block dot), acc)
        acc[0] = __fmaf_rn(__fmul_rn(dwa, dx0), (float)d[0], acc[0]);
        acc[1] = __fmaf_rn(__fmul_rn(dwa, dx1), (float)d[1], acc[1]);
        acc[2] = __fmaf_rn(__fmul_rn(dwb, dx0), (float)d[2], acc[2]);
        acc[3] = __fmaf_rn(__fmul_rn(dwb, dx1), (float)d[3], acc[3]);
    }
    part[warp][g][2 * t] = acc[0];
    part[warp][g][2 * t + 1] = acc[1];
    part[warp][g + 8][2 * t] = acc[2];
    part[warp][g + 8][2 * t + 1] = acc[3];
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < kRowsPerCta * 8; i += blockDim.x) {
        const uint32_t row = i / 8, col = i % 8;
        const int64_t r = r0 + row;
        if (r < rows && (int64_t)col < columns) {
            float v = ((part[0][row][col] + part[1][row][col]) + part[2][row][col]) + part[3][row][col];
            if (bias) v = __fadd_rn(v, bias[r - 0]);
            y[(int64_t)col * ldy + r] = v;
        }
    }
}

// ---------------------------------------------------------------- Q5_K ------

__device__ __forceinline__ void unpack_scales(const uint4 hdr, int (&sc)[8], int (&mn)[8])
{
    // bytes 4..15 of the super-block: the 12 packed 6-bit scales/mins
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    const uint8_t s[12] = {(uint8_t)s0, (uint8_t)(s0 >> 8), (uint8_t)(s0 >> 16), (uint8_t)(s0 >> 24),
                           (uint8_t)s1, (uint8_t)(s1 >> 8), (uint8_t)(s1 >> 16), (uint8_t)(s1 >> 24),
                           (uint8_t)s2, (uint8_t)(s2 >> 8), (uint8_t)(s2 >> 16), (uint8_t)(s2 >> 24)};
#pragma unroll
    for (int g = 0; g < 4; g++) {
        sc[g] = s[g] & 63;
        mn[g] = s[g + 4] & 63;
        sc[g + 4] = (s[g + 8] & 15) | ((s[g] >> 6) << 4);
        mn[g + 4] = (s[g + 8] >> 4) | ((s[g + 4] >> 6) << 4);
    }
}

__global__ void __launch_bounds__(128) k_matvec_q5_K(const uint8_t* __restrict__ w, int64_t stride, int64_t rows,
                                                     int64_t inner, const uint8_t* __restrict__ xq, int64_t columns,
                                                     float* __restrict__ y, int64_t ldy, const float* __restrict__ bias)
{
    __shared__ float part[kWarps][kRowsPerCta][8];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const int64_t r0 = (int64_t)blockIdx.x * kRowsPerCta;
    const int64_t ra = r0 + g, rb = r0 + g + 8;
    const bool va = ra < rows, vb = rb < rows;
    const int64_t nsb = inner / kQKK;
    const int64_t xstride = nsb * kQ8KBytes;
    const bool vx = (int64_t)g < columns;
    const uint8_t* wa = w + (va ? ra : 0) * stride;
    const uint8_t* wb = w + (vb ? rb : 0) * stride;
    const uint8_t* xr = xq + (vx ? g : 0) * xstride;
    const bool vc0 = (int64_t)(2 * t) < columns, vc1 = (int64_t)(2 * t + 1) < columns;
    const uint8_t* xc0 = xq + (vc0 ? 2 * t : 0) * xstride;
    const uint8_t* xc1 = xq + (vc1 ? 2 * t + 1 : 0) * xstride;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float summ[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t sb = warp; sb < nsb; sb += kWarps) {
        const uint8_t* ba = wa + sb * kQ5KBytes;
        const uint8_t* bb = wb + sb * kQ5KBytes;
        const uint8_t* bx = xr + sb * kQ8KBytes;
        const uint4 ha = va ? __ldg(reinterpret_cast<const uint4*>(ba)) : make_uint4(0, 0, 0, 0);
        const uint4 hb = vb ? __ldg(reinterpret_cast<const uint4*>(bb)) : make_uint4(0, 0, 0, 0);
        const uint2 qha = va ? __ldg(reinterpret_cast<const uint2*>(ba + 16 + 8 * t)) : make_uint2(0, 0);
        const uint2 qhb = vb ? __ldg(reinterpret_cast<const uint2*>(bb + 16 + 8 * t)) : make_uint2(0, 0);
        uint2 qsa[4], qsb[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            qsa[p] = va ? __ldg(reinterpret_cast<const uint2*>(ba + 48 + 32 * p + 8 * t)) : make_uint2(0, 0);
            qsb[p] = vb ? __ldg(reinterpret_cast<const uint2*>(bb + 48 + 32 * p + 8 * t)) : make_uint2(0, 0);
        }
        int sca[8], mna[8], scb[8], mnb[8];
        unpack_scales(ha, sca, mna);
        unpack_scales(hb, scb, mnb);
        int sumi[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int p = j / 2;
            const uint32_t sh = (j & 1) ? 4u : 0u;
            const uint32_t la0 = (qsa[p].x >> sh) & 0x0f0f0f0fu, la1 = (qsa[p].y >> sh) & 0x0f0f0f0fu;
            const uint32_t lb0 = (qsb[p].x >> sh) & 0x0f0f0f0fu, lb1 = (qsb[p].y >> sh) & 0x0f0f0f0fu;
            const uint32_t a[4] = {la0 | (((qha.x >> j) & 0x01010101u) << 4), lb0 | (((qhb.x >> j) & 0x01010101u) << 4),
                                   la1 | (((qha.y >> j) & 0x01010101u) << 4), lb1 | (((qhb.y >> j) & 0x01010101u) << 4)};
            uint32_t b0 = 0, b1 = 0;
            if (vx) {
                const uint32_t* q8 = reinterpret_cast<const uint32_t*>(bx + 4 + 32 * j + 8 * t);
                b0 = __ldg(q8);
                b1 = __ldg(q8 + 1);
            }
            int d[4];
            mma_s8(d, a, b0, b1);
            sumi[0] += sca[j] * d[0];
            sumi[1] += sca[j] * d[1];
            sumi[2] += scb[j] * d[2];
            sumi[3] += scb[j] * d[3];
        }
        // min term: sum_j m_j * (bsum_2j + bsum_2j+1) per (weight row, activation row)
        int msum[4] = {0, 0, 0, 0};
        const uint8_t* bx0 = xc0 + sb * kQ8KBytes;
        const uint8_t* bx1 = xc1 + sb * kQ8KBytes;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t p0 = vc0 ? __ldg(reinterpret_cast<const uint32_t*>(bx0 + 4 + kQKK + 4 * j)) : 0u;
            const uint32_t p1 = vc1 ? __ldg(reinterpret_cast<const uint32_t*>(bx1 + 4 + kQKK + 4 * j)) : 0u;
            const int s0 = (int)(int16_t)(p0 & 0xffffu) + (int)(int16_t)(p0 >> 16);
            const int s1 = (int)(int16_t)(p1 & 0xffffu) + (int)(int16_t)(p1 >> 16);
            msum[0] += mna[j] * s0;
            msum[1] += mna[j] * s1;
            msum[2] += mnb[j] * s0;
            msum[3] += mnb[j] * s1;
        }
        const float dx0 = vc0 ? __ldg(reinterpret_cast<const float*>(bx0)) : 0.f;
        const float dx1 = vc1 ? __ldg(reinterpret_cast<const float*>(bx1)) : 0.f;
        const float da = __half2float(__ushort_as_half((unsigned short)(ha.x & 0xffffu)));
        const float dma = __half2float(__ushort_as_half((unsigned short)(ha.x >> 16)));
        const float db = __half2float(__ushort_as_half((unsigned short)(hb.x & 0xffffu)));
        const float dmb = __half2float(__ushort_as_half((unsigned short)(hb.x >> 16)));
        // pix_dot_q5_K: d = y.d * fp16(x.d); dmin = -y.d * fp16(x.dmin)
        acc[0] = __fmaf_rn(__fmul_rn(dx0, da), (float)sumi[0], acc[0]);
        acc[1] = __fmaf_rn(__fmul_rn(dx1, da), (float)sumi[1], acc[1]);
        acc[2] = __fmaf_rn(__fmul_rn(dx0, db), (float)sumi[2], acc[2]);
        acc[3] = __fmaf_rn(__fmul_rn(dx1, db), (float)sumi[3], acc[3]);
        summ[0] = __fmaf_rn(__fmul_rn(-dx0, dma), (float)msum[0], summ[0]);
        summ[1] = __fmaf_rn(__fmul_rn(-dx1, dma), (float)msum[1], summ[1]);
        summ[2] = __fmaf_rn(__fmul_rn(-dx0, dmb), (float)msum[2], summ[2]);
        summ[3] = __fmaf_rn(__fmul_rn(-dx1, dmb), (float)msum[3], summ[3]);
    }
    part[warp][g][2 * t] = acc[0] + summ[0];
    part[warp][g][2 * t + 1] = acc[1] + summ[1];
    part[warp][g + 8][2 * t] = acc[2] + summ[2];
    part[warp][g + 8][2 * t + 1] = acc[3] + summ[3];
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < kRowsPerCta * 8; i += blockDim.x) {
        const uint32_t row = i / 8, col = i % 8;
        const int64_t r = r0 + row;
        if (r < rows && (int64_t)col < columns) {
            float v = ((part[0][row][col] + part[1][row][col]) + part[2][row][col]) + part[3][row][col];
            if (bias) v = __fadd_rn(v, bias[r]);
            y[(int64_t)col * ldy + r] = v;
        }
    }
}

}  // namespace

cudaError_t launch_matvec(uint32_t type, const uint8_t* w, int64_t stride, int64_t rows, int64_t inner, const void* xq,
                          int64_t columns, float* y, int64_t ldy, const float* bias, cudaStream_t s)
{
    if (columns < 1 || columns > 8) return cudaErrorInvalidValue;
    const int64_t ctas = (rows + kRowsPerCta - 1) / kRowsPerCta;
    if (ctas > 0x7fffffff) return cudaErrorInvalidValue;
    const uint8_t* x = static_cast<const uint8_t*>(xq);
    if (type == kTypeQ8_0) {
        k_matvec_q8_0<<<(unsigned)ctas, 128, 0, s>>>(w, stride, rows, inner, x, columns, y, ldy, bias);
    } else if (type == kTypeQ5_K) {
        k_matvec_q5_K<<<(unsigned)ctas, 128, 0, s>>>(w, stride, rows, inner, x, columns, y, ldy, bias);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace pxq
