// quantize.cu -- activation quantizers, bit-exact with Pixelina's CPU path.
//
//   Q8_0 (32-blocks)  restates quantize_row_q8_0_ref, src/kernels_quant.cpp:120-144
//   Q8_K (256-blocks) restates quantize_row_q8_K_ref, src/kernels_quant.cpp:80-118
//
// Each comes in several output layouts: the GGUF block layout (what the
// reference produces, checked by the parity tests; the Q8_0 matvec reads it
// too), the Q8_K matvec operand (the same bytes permuted for the matvec's
// fragments, plus 32-element sums), and the tensor-core operand layout used
// by the GEMM (the int8 quants, or exact fp16 copies of them, plus their
// block scales).  All layouts come from the same arithmetic.
//
// Bit-exactness rules (all arithmetic uses explicit _rn intrinsics so that
// nvcc's default FMA contraction cannot change a rounding):
//   * d = amax/127 and 1/d are IEEE divisions;
//   * Q8_0 rounds x*id half away from zero (roundf) after a rounded product
//     (q8_0_round in q8k.cuh: two round-toward-zero adds, no conversion
//     instruction);
//   * Q8_K rounds iscale*x half to even through the 1.5*2^23 bias, and the
//     reference build evaluates `iscale*x + bias` as ONE fused multiply-add
//     (g++ -O3 -std=c++17 contracts it; pinned by the golden vectors), so the
//     kernel uses __fmaf_rn for that step;
//   * the stored fp16 scale is round-to-nearest-even (F16C with
//     _MM_FROUND_TO_NEAREST_INT).
#include <atomic>

#include "pxq_device.cuh"
#include "pxq_internal.h"
#include "q8k.cuh"

namespace pxq {
namespace {

// One Q8_0 block per 2 consecutive threads, 16 elements per thread (the
// block's amax meets in one shuffle; a thread's fixed costs -- indexing, the
// two divisions, the stores -- are shared by 16 elements).
// Returns (d as stored fp16, the 16 quants, packed little-endian in 4 words).
struct Q80Part {
    __half d16;
    uint32_t packed[4];
    int q[16];
};

__device__ __forceinline__ Q80Part q8_0_part(const float4 (&v)[4])
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    Q80Part p;
    p.d16 = __float2half_rn(d);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        p.q[4 * i + 0] = q8_0_round(v[i].x, id);
        p.q[4 * i + 1] = q8_0_round(v[i].y, id);
        p.q[4 * i + 2] = q8_0_round(v[i].z, id);
        p.q[4 * i + 3] = q8_0_round(v[i].w, id);
        p.packed[i] = ((uint32_t)p.q[4 * i] & 0xffu) | (((uint32_t)p.q[4 * i + 1] & 0xffu) << 8) |
                      (((uint32_t)p.q[4 * i + 2] & 0xffu) << 16) | ((uint32_t)p.q[4 * i + 3] << 24);
    }
    return p;
}

// Start of every kernel that may run under programmatic stream serialization:
// let the next kernel launch, wait for the previous one, then clear the
// caller's counters (the matvec's split-K counters) if any.
__device__ __forceinline__ void pdl_prologue(uint32_t* __restrict__ zero, int64_t nzero)
{
    griddep_launch_dependents();
    griddep_wait();
    if (zero) {
        const int64_t cta = (int64_t)blockIdx.y * gridDim.x + blockIdx.x, nthr = (int64_t)gridDim.x * gridDim.y * blockDim.x;
        for (int64_t i = cta * blockDim.x + threadIdx.x; i < nzero; i += nthr) zero[i] = 0u;
    }
}

// The Q8_0 kernels walk a 2-D grid: x = groups of kQ80Threads consecutive
// 16-value halves of a row's blocks (2 threads per 32-block), y = a slab of
// rows taken kQ80Rows at a time (their loads all in flight before any block
// is reduced); no index divisions.  Threads past the row end compute on
// zeros and store nothing, so every shuffle has its full warp.
constexpr int kQ80Threads = 64;
constexpr int kQ80Rows = 2;

dim3 q8_0_grid(int64_t rows, int64_t inner)
{
    const int64_t gx = (inner / 16 + kQ80Threads - 1) / kQ80Threads;
    int64_t gy = (148 * 32 + gx - 1) / gx;  // about 32 CTAs per SM in all
    const int64_t max_gy = (rows + kQ80Rows - 1) / kQ80Rows;
    if (gy > max_gy) gy = max_gy;
    if (gy < 1) gy = 1;
    if (gy > 65535) gy = 65535;
    return dim3((unsigned)gx, (unsigned)gy);
}

// For every (row, half) of this thread: emit(row, half, part, valid); half h
// covers elements 16h .. 16h+15 of the row (block h / 2).  Every thread of
// the warp calls emit with the same row (valid is false past the row end or
// past the last row), so emitters may synchronise the warp.
template <typename Emit>
__device__ __forceinline__ void q8_0_rows(const float* x, int64_t rows, int64_t inner, int64_t ldx, Emit emit)
{
    const int64_t half = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool on = half < inner / 16;
    for (int64_t r0 = blockIdx.y; r0 < rows; r0 += (int64_t)kQ80Rows * gridDim.y) {
        float4 v[kQ80Rows][4];
#pragma unroll
        for (int u = 0; u < kQ80Rows; u++) {
            const int64_t r = r0 + (int64_t)u * gridDim.y;
#pragma unroll
            for (int i = 0; i < 4; i++)
                v[u][i] = on && r < rows ? ld_dep_f4(x + r * ldx + half * 16 + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kQ80Rows; u++) {
            const int64_t r = r0 + (int64_t)u * gridDim.y;
            const Q80Part p = q8_0_part(v[u]);
            emit(r, half, p, on && r < rows);
        }
    }
}

__global__ void k_quantize_q8_0_blocks(const float* x, uint8_t* __restrict__ y, int64_t rows, int64_t inner,
                                       int64_t ldx, uint32_t* __restrict__ zero, int64_t nzero)
{
    pdl_prologue(zero, nzero);
    const int64_t nb = inner / kQK8_0;
    // a warp's 16 consecutive 34-byte blocks are assembled in shared memory and
    // written out as consecutive 2-byte words (the blocks are only 2-byte
    // aligned), so every store instruction covers 64 contiguous bytes
    constexpr int kWords = 16 * kQ8_0Bytes / 2;
    __shared__ uint16_t stage[kQ80Threads / 32][kWords];
    const uint32_t lane = threadIdx.x & 31u;
    uint16_t* st = stage[threadIdx.x >> 5];
    const int64_t h0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31u);  // lane 0's half
    q8_0_rows(x, rows, inner, ldx, [&](int64_t row, int64_t half, const Q80Part& p, bool valid) {
        if (row >= rows) return;  // warp-uniform
        uint16_t* w16 = st + (lane >> 1) * (kQ8_0Bytes / 2);
        if (valid) {
            if ((lane & 1u) == 0) w16[0] = __half_as_ushort(p.d16);
#pragma unroll
            for (int w = 0; w < 4; w++) {
                w16[1 + 8 * (lane & 1u) + 2 * w] = (uint16_t)(p.packed[w] & 0xffffu);
                w16[2 + 8 * (lane & 1u) + 2 * w] = (uint16_t)(p.packed[w] >> 16);
            }
        }
        __syncwarp();
        int64_t nh = inner / 16 - h0;  // halves of this row from lane 0 on
        nh = nh < 0 ? 0 : (nh > 32 ? 32 : nh);
        const int words = (int)(nh / 2) * (kQ8_0Bytes / 2);
        uint16_t* dst = reinterpret_cast<uint16_t*>(y + (row * nb + h0 / 2) * kQ8_0Bytes);
        for (int i = (int)lane; i < words; i += 32) dst[i] = st[i];
        __syncwarp();
    });
}

// GEMM operand: the quants as int8 (kinds 1, 4) or exact fp16 values (kinds
// 0, 2), [rows][inner], and the stored fp16 block scales: as fp32,
// block-major [inner/32][ldd] (kinds 0, 1), or as fp16, row-major
// [rows][ldd] (kinds 2, 4).
__global__ void k_quantize_q8_0_operand(const float* __restrict__ x, void* __restrict__ xq, void* __restrict__ dx, int kind,
                                        int64_t rows, int64_t inner, int64_t ldx, int64_t ldd)
{
    q8_0_rows(x, rows, inner, ldx, [&](int64_t row, int64_t half, const Q80Part& p, bool valid) {
        if (!valid) return;
        if (kind == 1 || kind == 4) {
            *reinterpret_cast<uint4*>(static_cast<int8_t*>(xq) + row * inner + half * 16) =
                make_uint4(p.packed[0], p.packed[1], p.packed[2], p.packed[3]);
        } else {
            uint32_t h[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                __half2 v = small_int_half2(p.q[2 * i], p.q[2 * i + 1]);
                h[i] = *reinterpret_cast<uint32_t*>(&v);
            }
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(xq) + row * inner + half * 16);
            dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
            dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
        }
        if ((half & 1) == 0) {
            if (kind == 2 || kind == 4)
                static_cast<__half*>(dx)[row * ldd + half / 2] = p.d16;
            else
                static_cast<float*>(dx)[(half / 2) * ldd + row] = __half2float(p.d16);
        }
    });
}

// ---- Q8_K: one warp per 256-block (q8k.cuh) -------------------------------

// (row, super-block) of the warp's block index w, by 32-bit division (a 64-bit
// division costs several times more instructions than the block's own
// arithmetic; the launchers check that rows x super-blocks fits 32 bits)
__device__ __forceinline__ const float* q8_K_src(const float* x, int64_t w, uint32_t nsb, int64_t ldx, int64_t& row,
                                                 int64_t& sb)
{
    const uint32_t r = (uint32_t)w / nsb;
    row = r;
    sb = (uint32_t)w - r * nsb;
    return x + row * ldx + sb * kQKK;
}

// Matvec operand: one record per (row, super-block), kQ8KMvBytes for Q5_K
// weights (layout: q8_K_store_mv, q8k.cuh), kQ8KQ6Bytes for Q6_K weights
// (q8_K_store_q6).
template <bool Q6>
__global__ void k_quantize_q8_K_mv(const float* x, uint8_t* __restrict__ y, int64_t rows, int64_t inner,
                                   int64_t ldx, uint32_t* __restrict__ zero, int64_t nzero)
{
    pdl_prologue(zero, nzero);
    const uint32_t lane = threadIdx.x & 31u;
    const int64_t nsb = inner / kQKK;
    const int64_t total = rows * nsb;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t w = (((int64_t)blockIdx.x * blockDim.x) >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
        int64_t row, sb;
        const Q8KWarp r = q8_K_warp(q8_K_src(x, w, (uint32_t)nsb, ldx, row, sb), lane);
        if (Q6)
            q8_K_store_q6(y + w * kQ8KQ6Bytes, r, lane);
        else
            q8_K_store_mv(y + w * kQ8KMvBytes, r, lane);
    }
}

// Q8_0 activation rows as the streamed matvec's records: one warp per 256
// values (eight blocks), kQ80MvBytes each (q8_0_store_mv).
__global__ void k_quantize_q8_0_mv(const float* x, uint8_t* __restrict__ y, int64_t rows, int64_t inner, int64_t ldx,
                                   uint32_t* __restrict__ zero, int64_t nzero)
{
    pdl_prologue(zero, nzero);
    const uint32_t lane = threadIdx.x & 31u;
    const int64_t ngr = inner / kQKK;
    const int64_t total = rows * ngr;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t w = (((int64_t)blockIdx.x * blockDim.x) >> 5) + (threadIdx.x >> 5); w < total; w += warps) {
        float v[8];
        q8_K_load(x + (w / ngr) * ldx + (w % ngr) * kQKK, lane, v);
        q8_0_store_mv(y + w * kQ80MvBytes, v, lane);
    }
}

// One super-block per half warp, 16 values per lane (lanes 16h .. 16h+15
// hold the block's values 16*(lane%16) .. +15): the arithmetic of
// q8_K_warp_vals, with each warp's shuffles, ballot and divisions shared by two
// blocks.  Lanes of a half whose block is past the end compute on zeros.
struct Q8KHalf {
    float d;     // stored fp32 scale (1/iscale, or 0 for an all-zero block)
    int q[16];   // this lane's 16 quants
};

__device__ __forceinline__ Q8KHalf q8_K_half_vals(const float (&v)[16], uint32_t lane)
{
    // first element (in index order) with the largest |x|: the half's largest
    // |x| (NaNs never win), then the lowest lane of the half holding it
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float vsel = 0.0f;
    bool hit = false;
#pragma unroll
    for (int j = 15; j >= 0; j--) {
        if (fabsf(v[j]) == amax) {
            vsel = v[j];
            hit = true;
        }
    }
    const uint32_t half_mask = (lane & 16u) ? 0xffff0000u : 0x0000ffffu;
    const uint32_t hits = __ballot_sync(0xffffffffu, hit) & half_mask;
    const float vmax = __shfl_sync(0xffffffffu, vsel, hits ? __ffs(hits) - 1 : (int)(lane & 16u));
    Q8KHalf r;
    if (amax == 0.0f) {
        r.d = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; j++) r.q[j] = 0;
        return r;
    }
    const float iscale = __fdiv_rn(-127.0f, vmax);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const float biased = __fmaf_rn(iscale, v[j], 12582912.0f);
        const int bits = __float_as_int(biased);
        const int q = (bits & 0x007fffff) - 0x00400000;
        r.q[j] = (int8_t)(q < 127 ? q : 127);
    }
    r.d = __fdiv_rn(1.0f, iscale);
    return r;
}

// GGUF Q8_K blocks {f32 d; int8 qs[256]; int16 bsums[16]}: one block per half
// warp; lane l of a half writes quants 16l .. 16l+15 (4-byte stores: the
// 292-byte blocks are 4-byte aligned) and their sum, which is bsums[l].
__global__ void k_quantize_q8_K_blocks(const float* __restrict__ x, uint8_t* __restrict__ y, int64_t rows, int64_t inner,
                                       int64_t ldx)
{
    const uint32_t lane = threadIdx.x & 31u, hl = lane & 15u;
    const int64_t nsb = inner / kQKK;
    const int64_t total = rows * nsb;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t wb = 2 * ((((int64_t)blockIdx.x * blockDim.x) >> 5) + (threadIdx.x >> 5)); wb < total; wb += 2 * warps) {
        const int64_t w = wb + (lane >> 4);
        const bool valid = w < total;  // uniform within the half
        float v[16];
        if (valid) {
            int64_t row, sb;
            const float* src = q8_K_src(x, w, (uint32_t)nsb, ldx, row, sb) + hl * 16;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 f = ld_dep_f4(src + 4 * i);
                v[4 * i] = f.x;
                v[4 * i + 1] = f.y;
                v[4 * i + 2] = f.z;
                v[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = 0.0f;
        }
        const Q8KHalf r = q8_K_half_vals(v, lane);
        if (valid) {
            uint8_t* out = y + w * kQ8KBytes;
            uint32_t* qs = reinterpret_cast<uint32_t*>(out + 4 + hl * 16);
            int sum16 = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                qs[i] = ((uint32_t)r.q[4 * i] & 0xffu) | (((uint32_t)r.q[4 * i + 1] & 0xffu) << 8) |
                        (((uint32_t)r.q[4 * i + 2] & 0xffu) << 16) | ((uint32_t)r.q[4 * i + 3] << 24);
                sum16 += r.q[4 * i] + r.q[4 * i + 1] + r.q[4 * i + 2] + r.q[4 * i + 3];
            }
            *reinterpret_cast<int16_t*>(out + 4 + kQKK + 2 * hl) = (int16_t)sum16;
            if (hl == 0) *reinterpret_cast<float*>(out) = r.d;
        }
    }
}

// GEMM operand of the K-quant kernels: exact fp16 quants [rows][inner], the
// fp32 scales block-major [inner/256][ldd], and each 32-element sum split as
// (floor(s/64), s mod 64) in fp16 [rows][inner/256 * 16].  Two super-blocks
// per warp (one per half).
__global__ void k_quantize_q8_K_operand(const float* __restrict__ x, __half* __restrict__ xq, float* __restrict__ dxT,
                                        __half* __restrict__ amin, int64_t rows, int64_t inner, int64_t ldx, int64_t ldd)
{
    const uint32_t lane = threadIdx.x & 31u, hl = lane & 15u;
    const int64_t nsb = inner / kQKK;
    const int64_t total = rows * nsb;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t wb = 2 * ((((int64_t)blockIdx.x * blockDim.x) >> 5) + (threadIdx.x >> 5)); wb < total; wb += 2 * warps) {
        const int64_t w = wb + (lane >> 4);
        const bool valid = w < total;  // uniform within the half
        float v[16];
        int64_t row = 0, sb = 0;
        if (valid) {
            const float* src = q8_K_src(x, w, (uint32_t)nsb, ldx, row, sb) + hl * 16;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 f = ld_dep_f4(src + 4 * i);
                v[4 * i] = f.x;
                v[4 * i + 1] = f.y;
                v[4 * i + 2] = f.z;
                v[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = 0.0f;
        }
        const Q8KHalf r = q8_K_half_vals(v, lane);
        int sum16 = 0;
#pragma unroll
        for (int j = 0; j < 16; j++) sum16 += r.q[j];
        const int s32 = sum16 + __shfl_xor_sync(0xffffffffu, sum16, 1);  // 32-element sub-block = lane pair
        if (valid) {
            uint32_t h[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                __half2 p2 = small_int_half2(r.q[2 * i], r.q[2 * i + 1]);
                h[i] = *reinterpret_cast<uint32_t*>(&p2);
            }
            uint4* dst = reinterpret_cast<uint4*>(xq + row * inner + sb * kQKK + hl * 16);
            dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
            dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
            if ((hl & 1u) == 0) {
                const int j = (int)(hl >> 1);
                const int hi = s32 >> 6;         // floor(s32 / 64)
                const int lo = s32 - (hi << 6);  // 0..63
                __half2 pair = small_int_half2(hi, lo);
                *reinterpret_cast<__half2*>(amin + row * (nsb * 16) + sb * 16 + 2 * j) = pair;
            }
            if (hl == 0) dxT[sb * ldd + row] = r.d;
        }
    }
}

int grid_for(int64_t work_items, int threads)
{
    int64_t blocks = (work_items + threads - 1) / threads;
    if (blocks < 1) blocks = 1;
    if (blocks > 148 * 64) blocks = 148 * 64;
    return (int)blocks;
}

// Q6_K rows for the device: every 210-byte super-block padded to 224 bytes
// (16-byte multiples, as TMA rows need); bytes 210..223 are zero.
__global__ void k_pad_q6_K(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int64_t superblocks)
{
    const int64_t total = superblocks * (kQ6KPadBytes / 2);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t sb = i / (kQ6KPadBytes / 2), e = i % (kQ6KPadBytes / 2);
        dst[i] = e < kQ6KBytes / 2 ? src[sb * (kQ6KBytes / 2) + e] : (uint16_t)0;
    }
}

}  // namespace

cudaError_t launch_pad_q6_K(const void* src, void* dst, int64_t superblocks, cudaStream_t s)
{
    const int threads = 256;
    k_pad_q6_K<<<grid_for(superblocks * (kQ6KPadBytes / 2), threads), threads, 0, s>>>(static_cast<const uint16_t*>(src),
                                                                                     static_cast<uint16_t*>(dst), superblocks);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0_blocks(const float* x, void* y, int64_t rows, int64_t inner, int64_t ldx, cudaStream_t s)
{
    k_quantize_q8_0_blocks<<<q8_0_grid(rows, inner), kQ80Threads, 0, s>>>(x, static_cast<uint8_t*>(y), rows, inner, ldx,
                                                                          nullptr, 0);
    return cudaGetLastError();
}

cudaError_t launch_matvec_quantize(const MatvecPlan& plan, const float* x, int64_t ldx, void* act, uint32_t* counters,
                                   cudaStream_t s)
{
    const int threads = 256;
    const int64_t nzero = counters ? (int64_t)(plan.counter_bytes / 4) : 0;
    uint8_t* out = static_cast<uint8_t*>(act);
    if (plan.type == kTypeQ8_0 && plan.streamed)
        return launch_pdl(k_quantize_q8_0_mv, dim3(grid_for(plan.columns * (plan.inner / kQKK) * 32, threads)), dim3(threads), 0, s,
                          x, out, plan.columns, plan.inner, ldx, counters, nzero);
    if (plan.type == kTypeQ8_0)
        return launch_pdl(k_quantize_q8_0_blocks, q8_0_grid(plan.columns, plan.inner), dim3(kQ80Threads), 0, s,
                          x, out, plan.columns, plan.inner, ldx, counters, nzero);
    if (plan.type == kTypeQ5_K || plan.type == kTypeQ6_K) {
        const bool q6 = plan.type == kTypeQ6_K;
        auto kern = q6 ? k_quantize_q8_K_mv<true> : k_quantize_q8_K_mv<false>;
        // same shared-memory carveout as the matvec, so that the SMs need no
        // reconfiguration between the two kernels
        // (set once per device; setting it twice from racing threads is harmless)
        static std::atomic<bool> carveout_set[2][16] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 0 && dev < 16 && !carveout_set[q6][dev].load(std::memory_order_acquire)) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                 (int)cudaSharedmemCarveoutMaxShared);
            if (e != cudaSuccess) return e;
            carveout_set[q6][dev].store(true, std::memory_order_release);
        }
        return launch_pdl(kern, dim3(grid_for(plan.columns * (plan.inner / kQKK) * 32, threads)), dim3(threads), 0, s, x, out,
                          plan.columns, plan.inner, ldx, counters, nzero);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_quantize_q8_K_blocks(const float* x, void* y, int64_t rows, int64_t inner, int64_t ldx, cudaStream_t s)
{
    const int threads = 256;
    if (rows * (inner / kQKK) >= (int64_t)1 << 31) return cudaErrorInvalidValue;
    k_quantize_q8_K_blocks<<<grid_for(rows * (inner / kQKK) * 16, threads), threads, 0, s>>>(x, static_cast<uint8_t*>(y), rows,
                                                                                            inner, ldx);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0_operand(const float* x, void* xq, void* dx, int kind, int64_t rows, int64_t inner,
                                         int64_t ldx, int64_t ldd, cudaStream_t s)
{
    k_quantize_q8_0_operand<<<q8_0_grid(rows, inner), kQ80Threads, 0, s>>>(x, xq, dx, kind, rows, inner, ldx, ldd);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_K_operand(const float* x, __half* xq, float* dxT, __half* amin, int64_t rows, int64_t inner,
                                         int64_t ldx, int64_t ldd, cudaStream_t s)
{
    const int threads = 256;
    if (rows * (inner / kQKK) >= (int64_t)1 << 31) return cudaErrorInvalidValue;
    k_quantize_q8_K_operand<<<grid_for(rows * (inner / kQKK) * 16, threads), threads, 0, s>>>(x, xq, dxT, amin, rows, inner,
                                                                                             ldx, ldd);
    return cudaGetLastError();
}

}  // namespace pxq
