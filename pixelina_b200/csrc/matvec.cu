// matvec.cu -- small-M (decode) quantized matvec: y = X * W^T for M <= 8.
//
// Restates, for columns <= 8, the inner loop of cpu_quant_matmul
// (src/kernels_quant.cpp:389-400) with the dots pix_dot_q8_0 (:339-365) and
// pix_dot_q5_K (:163-254) on GPU: activations are the reference's Q8_0 /
// Q8_K blocks (produced by quantize.cu), weights stream straight from the raw
// GGUF rows in HBM.
//
// Mapping.  A CTA of 4 warps owns 16 weight rows and a range of K blocks
// (the whole row, or a 1/ks slice when there are too few row groups to fill
// the GPU -- split-K).  Its warps walk the K blocks round-robin, each with the
// next block's weight bytes already in flight (register double buffering);
// the small activation blocks are read through L1, shared by all CTAs.
// Each 32-value block is one int8 tensor-core mma.sync m16n8k32: A = the 16
// weight rows unpacked in registers, B = the up-to-8 activation rows
// (n = activation row, zero-padded), so one weight fragment serves all rows.
// The exact int32 block dot comes out of the MMA; the per-block fp32 scaling
// and the Q5_K sub-block scales / min term are applied in registers exactly
// as the reference does (int32 super-block sums, then one fp32 FMA per
// super-block).  The K order inside a 32-block is permuted identically for A
// and B (a dot product does not depend on the order of its terms) so that
// each thread's 8 weight bytes per block are contiguous in memory.
// Partials of the 4 warps are summed in shared memory in fixed order; with
// split-K the slices are summed, again in fixed order, by the last CTA of the
// row group to finish.  Results are therefore deterministic.
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int kRowsPerCta = 16;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// 8 bytes from a 2-byte-aligned address (Q8_0 blocks are 34 bytes).
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

// Cross-warp sum (fixed order), then either the final store or the split-K
// partial and, for the last CTA of the row group, the fixed-order reduction.
__device__ __forceinline__ void finish(float (&part)[kWarps][kRowsPerCta][8], int64_t r0, int64_t rows, int64_t columns,
                                       float* __restrict__ y, int64_t ldy, const float* __restrict__ bias, int ks, int kc,
                                       int64_t rg, float* __restrict__ partial, uint32_t* __restrict__ counters)
{
    __shared__ int s_last;
    __syncthreads();
    if (ks == 1) {
        for (uint32_t i = threadIdx.x; i < kRowsPerCta * 8; i += kThreads) {
            const uint32_t row = i / 8, col = i % 8;
            const int64_t r = r0 + row;
            if (r < rows && (int64_t)col < columns) {
                float v = ((part[0][row][col] + part[1][row][col]) + part[2][row][col]) + part[3][row][col];
                if (bias) v = __fadd_rn(v, bias[r]);
                y[(int64_t)col * ldy + r] = v;
            }
        }
        return;
    }
    for (uint32_t i = threadIdx.x; i < kRowsPerCta * 8; i += kThreads) {
        const uint32_t row = i / 8, col = i % 8;
        const int64_t r = r0 + row;
        if (r < rows && (int64_t)col < columns)
            partial[((int64_t)kc * columns + col) * rows + r] =
                ((part[0][row][col] + part[1][row][col]) + part[2][row][col]) + part[3][row][col];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[rg], 1u) == (uint32_t)(ks - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (uint32_t i = threadIdx.x; i < kRowsPerCta * 8; i += kThreads) {
        const uint32_t row = i / 8, col = i % 8;
        const int64_t r = r0 + row;
        if (r < rows && (int64_t)col < columns) {
            float v = 0.f;
            for (int k = 0; k < ks; k++) v += __ldcg(&partial[((int64_t)k * columns + col) * rows + r]);
            if (bias) v = __fadd_rn(v, bias[r]);
            y[(int64_t)col * ldy + r] = v;
        }
    }
    if (threadIdx.x == 0) counters[rg] = 0u;  // leave the counter ready for the next call
}

// ---------------------------------------------------------------- Q8_0 ------

__global__ void __launch_bounds__(kThreads) k_matvec_q8_0(const uint8_t* __restrict__ w, int64_t stride, int64_t rows,
                                                          int64_t inner, const uint8_t* __restrict__ xq, int64_t columns,
                                                          float* __restrict__ y, int64_t ldy, const float* __restrict__ bias,
                                                          int ks, int chunk, float* __restrict__ partial,
                                                          uint32_t* __restrict__ counters)
{
    __shared__ float part[kWarps][kRowsPerCta][8];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const int64_t rg = blockIdx.x / ks;
    const int kc = (int)(blockIdx.x % ks);
    const int64_t r0 = rg * kRowsPerCta;
    const int64_t nb = inner / kQK8_0;
    const int64_t b0 = (int64_t)kc * chunk, b1 = min(nb, b0 + chunk);
    const int64_t xstride = nb * kQ8_0Bytes;
    const int64_t ra = r0 + g, rb = r0 + g + 8;
    const bool va = ra < rows, vb = rb < rows;
    const bool vx = (int64_t)g < columns;  // B column n = g is activation row g
    const uint8_t* wa = w + (va ? ra : 0) * stride;
    const uint8_t* wb = w + (vb ? rb : 0) * stride;
    // activation blocks are small and shared by every CTA: read through L1
    const uint8_t* xr = xq + (vx ? g : 0) * xstride + b0 * kQ8_0Bytes;
    // this thread's two output columns (activation rows) are 2t and 2t+1
    const uint8_t* xc0 = xq + min((int64_t)(2 * t), columns - 1) * xstride + b0 * kQ8_0Bytes;
    const uint8_t* xc1 = xq + min((int64_t)(2 * t + 1), columns - 1) * xstride + b0 * kQ8_0Bytes;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int64_t b = b0 + warp;
    uint2 qa = make_uint2(0, 0), qb = make_uint2(0, 0);
    float dwa = 0.f, dwb = 0.f;
    if (b < b1) {
        if (va) { qa = ld8_unaligned(wa + b * kQ8_0Bytes + 2 + 8 * t); dwa = ld_half(wa + b * kQ8_0Bytes); }
        if (vb) { qb = ld8_unaligned(wb + b * kQ8_0Bytes + 2 + 8 * t); dwb = ld_half(wb + b * kQ8_0Bytes); }
    }
    for (; b < b1; b += kWarps) {
        // next block's weights in flight while this one computes
        uint2 na = make_uint2(0, 0), nbv = make_uint2(0, 0);
        float ndwa = 0.f, ndwb = 0.f;
        const int64_t bn = b + kWarps;
        if (bn < b1) {
            if (va) { na = ld8_unaligned(wa + bn * kQ8_0Bytes + 2 + 8 * t); ndwa = ld_half(wa + bn * kQ8_0Bytes); }
            if (vb) { nbv = ld8_unaligned(wb + bn * kQ8_0Bytes + 2 + 8 * t); ndwb = ld_half(wb + bn * kQ8_0Bytes); }
        }
        const int64_t off = (b - b0) * kQ8_0Bytes;
        const uint2 qx = vx ? ld8_unaligned(xr + off + 2 + 8 * t) : make_uint2(0, 0);
        const uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
        int d[4];
        mma_s8(d, a, qx.x, qx.y);
        const float dx0 = ld_half(xc0 + off), dx1 = ld_half(xc1 + off);
        // pix_dot_q8_0: acc = fma(fp16(dw) * fp16(dx), float(block dot), acc)
        acc[0] = __fmaf_rn(__fmul_rn(dwa, dx0), (float)d[0], acc[0]);
        acc[1] = __fmaf_rn(__fmul_rn(dwa, dx1), (float)d[1], acc[1]);
        acc[2] = __fmaf_rn(__fmul_rn(dwb, dx0), (float)d[2], acc[2]);
        acc[3] = __fmaf_rn(__fmul_rn(dwb, dx1), (float)d[3], acc[3]);
        qa = na;
        qb = nbv;
        dwa = ndwa;
        dwb = ndwb;
    }
    part[warp][g][2 * t] = acc[0];
    part[warp][g][2 * t + 1] = acc[1];
    part[warp][g + 8][2 * t] = acc[2];
    part[warp][g + 8][2 * t + 1] = acc[3];
    finish(part, r0, rows, columns, y, ldy, bias, ks, kc, rg, partial, counters);
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

// One thread's share of a super-block of its two weight rows (g and g+8).
struct Q5Frag {
    uint4 ha, hb;      // d, dmin, scales
    uint2 qha, qhb;    // high bits, bytes 8t..8t+7
    uint2 qsa[4], qsb[4];
};

__device__ __forceinline__ void load_q5(Q5Frag& f, const uint8_t* ba, const uint8_t* bb, bool va, bool vb, uint32_t t)
{
    f.ha = va ? __ldg(reinterpret_cast<const uint4*>(ba)) : make_uint4(0, 0, 0, 0);
    f.hb = vb ? __ldg(reinterpret_cast<const uint4*>(bb)) : make_uint4(0, 0, 0, 0);
    f.qha = va ? __ldg(reinterpret_cast<const uint2*>(ba + 16 + 8 * t)) : make_uint2(0, 0);
    f.qhb = vb ? __ldg(reinterpret_cast<const uint2*>(bb + 16 + 8 * t)) : make_uint2(0, 0);
#pragma unroll
    for (int p = 0; p < 4; p++) {
        f.qsa[p] = va ? __ldg(reinterpret_cast<const uint2*>(ba + 48 + 32 * p + 8 * t)) : make_uint2(0, 0);
        f.qsb[p] = vb ? __ldg(reinterpret_cast<const uint2*>(bb + 48 + 32 * p + 8 * t)) : make_uint2(0, 0);
    }
}

__global__ void __launch_bounds__(kThreads) k_matvec_q5_K(const uint8_t* __restrict__ w, int64_t stride, int64_t rows,
                                                          int64_t inner, const uint8_t* __restrict__ xq, int64_t columns,
                                                          float* __restrict__ y, int64_t ldy, const float* __restrict__ bias,
                                                          int ks, int chunk, float* __restrict__ partial,
                                                          uint32_t* __restrict__ counters)
{
    __shared__ float part[kWarps][kRowsPerCta][8];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const int64_t rg = blockIdx.x / ks;
    const int kc = (int)(blockIdx.x % ks);
    const int64_t r0 = rg * kRowsPerCta;
    const int64_t nsb = inner / kQKK;
    const int64_t s0 = (int64_t)kc * chunk, s1 = min(nsb, s0 + chunk);
    const int64_t ra = r0 + g, rb = r0 + g + 8;
    const bool va = ra < rows, vb = rb < rows;
    const bool vx = (int64_t)g < columns;
    const uint8_t* wa = w + (va ? ra : 0) * stride;
    const uint8_t* wb = w + (vb ? rb : 0) * stride;
    // activation blocks are small and shared by every CTA: read through L1
    const int64_t cstride = nsb * kQ8KBytes;
    const uint8_t* xr = xq + (vx ? g : 0) * cstride + s0 * kQ8KBytes;
    const bool vc0 = (int64_t)(2 * t) < columns, vc1 = (int64_t)(2 * t + 1) < columns;
    const uint8_t* xc0 = xq + (vc0 ? 2 * t : 0) * cstride + s0 * kQ8KBytes;
    const uint8_t* xc1 = xq + (vc1 ? 2 * t + 1 : 0) * cstride + s0 * kQ8KBytes;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float summ[4] = {0.f, 0.f, 0.f, 0.f};
    int64_t sb = s0 + warp;
    Q5Frag cur;
    if (sb < s1) load_q5(cur, wa + sb * kQ5KBytes, wb + sb * kQ5KBytes, va, vb, t);
    for (; sb < s1; sb += kWarps) {
        // next super-block's weights in flight while this one computes
        Q5Frag nxt;
        const int64_t sn = sb + kWarps;
        if (sn < s1) load_q5(nxt, wa + sn * kQ5KBytes, wb + sn * kQ5KBytes, va, vb, t);
        const uint8_t* bx = xr + (sb - s0) * kQ8KBytes;
        int sca[8], mna[8], scb[8], mnb[8];
        unpack_scales(cur.ha, sca, mna);
        unpack_scales(cur.hb, scb, mnb);
        int sumi[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int p = j / 2;
            const uint32_t sh = (j & 1) ? 4u : 0u;
            const uint32_t la0 = (cur.qsa[p].x >> sh) & 0x0f0f0f0fu, la1 = (cur.qsa[p].y >> sh) & 0x0f0f0f0fu;
            const uint32_t lb0 = (cur.qsb[p].x >> sh) & 0x0f0f0f0fu, lb1 = (cur.qsb[p].y >> sh) & 0x0f0f0f0fu;
            const uint32_t a[4] = {la0 | (((cur.qha.x >> j) & 0x01010101u) << 4),
                                   lb0 | (((cur.qhb.x >> j) & 0x01010101u) << 4),
                                   la1 | (((cur.qha.y >> j) & 0x01010101u) << 4),
                                   lb1 | (((cur.qhb.y >> j) & 0x01010101u) << 4)};
            uint32_t bq0 = 0, bq1 = 0;
            if (vx) {
                const uint32_t* q8 = reinterpret_cast<const uint32_t*>(bx + 4 + 32 * j + 8 * t);
                bq0 = __ldg(q8);
                bq1 = __ldg(q8 + 1);
            }
            int d[4];
            mma_s8(d, a, bq0, bq1);
            sumi[0] += sca[j] * d[0];
            sumi[1] += sca[j] * d[1];
            sumi[2] += scb[j] * d[2];
            sumi[3] += scb[j] * d[3];
        }
        // min term: sum_j m_j * (bsum_2j + bsum_2j+1) per (weight row, activation row)
        int msum[4] = {0, 0, 0, 0};
        const uint8_t* bx0 = xc0 + (sb - s0) * kQ8KBytes;
        const uint8_t* bx1 = xc1 + (sb - s0) * kQ8KBytes;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t p0 = vc0 ? __ldg(reinterpret_cast<const uint32_t*>(bx0 + 4 + kQKK + 4 * j)) : 0u;
            const uint32_t p1 = vc1 ? __ldg(reinterpret_cast<const uint32_t*>(bx1 + 4 + kQKK + 4 * j)) : 0u;
            const int q0 = (int)(int16_t)(p0 & 0xffffu) + (int)(int16_t)(p0 >> 16);
            const int q1 = (int)(int16_t)(p1 & 0xffffu) + (int)(int16_t)(p1 >> 16);
            msum[0] += mna[j] * q0;
            msum[1] += mna[j] * q1;
            msum[2] += mnb[j] * q0;
            msum[3] += mnb[j] * q1;
        }
        const float dx0 = vc0 ? __ldg(reinterpret_cast<const float*>(bx0)) : 0.f;
        const float dx1 = vc1 ? __ldg(reinterpret_cast<const float*>(bx1)) : 0.f;
        const float da = __half2float(__ushort_as_half((unsigned short)(cur.ha.x & 0xffffu)));
        const float dma = __half2float(__ushort_as_half((unsigned short)(cur.ha.x >> 16)));
        const float db = __half2float(__ushort_as_half((unsigned short)(cur.hb.x & 0xffffu)));
        const float dmb = __half2float(__ushort_as_half((unsigned short)(cur.hb.x >> 16)));
        // pix_dot_q5_K: d = y.d * fp16(x.d); dmin = -y.d * fp16(x.dmin)
        acc[0] = __fmaf_rn(__fmul_rn(dx0, da), (float)sumi[0], acc[0]);
        acc[1] = __fmaf_rn(__fmul_rn(dx1, da), (float)sumi[1], acc[1]);
        acc[2] = __fmaf_rn(__fmul_rn(dx0, db), (float)sumi[2], acc[2]);
        acc[3] = __fmaf_rn(__fmul_rn(dx1, db), (float)sumi[3], acc[3]);
        summ[0] = __fmaf_rn(__fmul_rn(-dx0, dma), (float)msum[0], summ[0]);
        summ[1] = __fmaf_rn(__fmul_rn(-dx1, dma), (float)msum[1], summ[1]);
        summ[2] = __fmaf_rn(__fmul_rn(-dx0, dmb), (float)msum[2], summ[2]);
        summ[3] = __fmaf_rn(__fmul_rn(-dx1, dmb), (float)msum[3], summ[3]);
        if (sn < s1) cur = nxt;
    }
    part[warp][g][2 * t] = acc[0] + summ[0];
    part[warp][g][2 * t + 1] = acc[1] + summ[1];
    part[warp][g + 8][2 * t] = acc[2] + summ[2];
    part[warp][g + 8][2 * t + 1] = acc[3] + summ[3];
    finish(part, r0, rows, columns, y, ldy, bias, ks, kc, rg, partial, counters);
}

}  // namespace

MatvecPlan plan_matvec(uint32_t type, int64_t rows, int64_t inner, int64_t columns, int num_sms)
{
    MatvecPlan p;
    const int64_t nblocks = type == kTypeQ8_0 ? inner / kQK8_0 : inner / kQKK;
    const int64_t min_chunk = type == kTypeQ8_0 ? 32 : 4;  // keep every warp busy on a slice
    p.rowgroups = (rows + kRowsPerCta - 1) / kRowsPerCta;
    // enough CTAs to cover every SM a few times, and an activation slice that fits the staging budget
    const int64_t target = (int64_t)num_sms * 4;
    int64_t ks = (target + p.rowgroups - 1) / p.rowgroups;
    const int64_t max_ks_work = nblocks / min_chunk > 1 ? nblocks / min_chunk : 1;
    if (ks > max_ks_work) ks = max_ks_work;
    if (ks < 1) ks = 1;
    const int64_t chunk = (nblocks + ks - 1) / ks;
    ks = (nblocks + chunk - 1) / chunk;
    p.ks = (int)ks;
    p.chunk = (int)chunk;
    p.smem_bytes = 0;
    p.partial_bytes = ks > 1 ? (size_t)ks * columns * rows * sizeof(float) : 0;
    p.counter_bytes = ks > 1 ? (size_t)p.rowgroups * sizeof(uint32_t) : 0;
    return p;
}

cudaError_t launch_matvec(uint32_t type, const uint8_t* w, int64_t stride, int64_t rows, int64_t inner, const void* xq,
                          int64_t columns, float* y, int64_t ldy, const float* bias, const MatvecPlan& plan, float* partial,
                          uint32_t* counters, cudaStream_t s)
{
    if (columns < 1 || columns > 8) return cudaErrorInvalidValue;
    const int64_t ctas = plan.rowgroups * plan.ks;
    if (ctas > 0x7fffffff || ctas < 1) return cudaErrorInvalidValue;
    if (plan.ks > 1 && (!partial || !counters)) return cudaErrorInvalidValue;
    const uint8_t* x = static_cast<const uint8_t*>(xq);
    if (type == kTypeQ8_0) {
        k_matvec_q8_0<<<(unsigned)ctas, kThreads, plan.smem_bytes, s>>>(w, stride, rows, inner, x, columns, y, ldy, bias,
                                                                        plan.ks, plan.chunk, partial, counters);
    } else if (type == kTypeQ5_K) {
        k_matvec_q5_K<<<(unsigned)ctas, kThreads, plan.smem_bytes, s>>>(w, stride, rows, inner, x, columns, y, ldy, bias,
                                                                        plan.ks, plan.chunk, partial, counters);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace pxq
