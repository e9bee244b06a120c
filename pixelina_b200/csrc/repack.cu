// repack.cu -- weight unpack kernels.
//
// (1) One-time repack of raw GGUF weight rows into the GEMM operand layout,
//     done when a weight is first used by the GEMM and then cached with it
//     (the device-side counterpart of the Vulkan backend's upload cache,
//     src/backend_vulkan.cpp:742-758):
//       Q8_0: wq   [rows][inner] = the int8 quants, as stored (operand kind
//                  1) or as exact fp16 values (kinds 0, 2)
//             dT   fp32 [inner/32][ldn] = the fp16 block scales, block-major
//                  (kinds 0, 1); kind 2: ws1h fp16 [rows][inner/32*16], the
//                  one-hot weight side of the tensor-core scale product
//       Q5_K: wv   fp16 [rows][inner]   = sc_g * q5 (<= 63*31 = 1953, exact)
//             dT, dminT fp32 [inner/256][ldn]
//             bmin fp16 [rows][inner/256*16] = (64*m_g, m_g) pairs, the weight
//                  side of the exact min-term product
//       Q6_K: wab  fp16 [rows][2*inner]: v = sc*(q6-32) (src/kernels_quant.cpp:
//                  256-337 folded per value) split into an even part a = v & ~1
//                  (|a| <= 4096, exact in fp16) and a parity part b = v & 1, so
//                  that a + b = v exactly; per 64-value chunk c, a fills
//                  [128c, 128c+64) and b [128c+64, 128c+128)
//             dT   fp32 [inner/256][ldn]
//     The bit layouts read here are those of src/backend_cpu.cpp:92-120
//     (cpu_decode) and src/kernels_quant.cpp:18-23 / 189-194.
// (2) pxq decode: dequantize to fp32 exactly as cpu_decode does
//     (src/backend_cpu.cpp:24-101), evaluation order included.
#include "pxq_internal.h"

namespace pxq {
namespace {

__device__ __forceinline__ void k_scale_min(const uint8_t* s, int g, int& sc, int& mn)
{
    if (g < 4) {
        sc = s[g] & 63;
        mn = s[g + 4] & 63;
    } else {
        sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
        mn = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
    }
}

__device__ __forceinline__ float load_half(const uint8_t* p)
{
    const uint16_t bits = (uint16_t)p[0] | ((uint16_t)p[1] << 8);
    return __half2float(__ushort_as_half(bits));
}

// Raw row behind packed operand row r.  gate_rows = 0: r itself.  A gated
// weight (F = gate_rows gate rows, then F up rows) packs as 128-row groups of
// 64 gate rows and the 64 matching up rows, so that each GEMM CTA tile holds
// both halves of its outputs.
__device__ __forceinline__ int64_t src_row(int64_t r, int64_t gate_rows)
{
    if (!gate_rows) return r;
    const int64_t j = r >> 7, q = r & 127;
    return q < 64 ? 64 * j + q : gate_rows + 64 * j + (q - 64);
}

// One thread per (row, 32-block): the block's 32 quants into the operand row
// (int8 as stored for kinds 1 and 4, their exact fp16 values otherwise) and
// its fp16 scale into the block-major fp32 plane (kinds 0, 1) or the one-hot
// tile (kinds 2, 4).
__global__ void k_repack_q8_0(const uint8_t* __restrict__ raw, int64_t rows, int64_t inner, int64_t stride,
                              void* __restrict__ wq, float* __restrict__ dT, __half* __restrict__ ws1h, int64_t ldn, int kind,
                              int64_t gate_rows)
{
    const int64_t nb = inner / kQK8_0;
    const int64_t total = rows * nb;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nb, b = i % nb;
        const uint8_t* blk = raw + src_row(r, gate_rows) * stride + b * kQ8_0Bytes;
        if (kind == 1 || kind == 4) {
            // qs start at byte 2 of the 34-byte block: 2-byte aligned loads
            uint16_t q[16];
#pragma unroll
            for (int j = 0; j < 16; j++) q[j] = reinterpret_cast<const uint16_t*>(blk + 2)[j];
            uint4* dst = reinterpret_cast<uint4*>(static_cast<int8_t*>(wq) + r * inner + b * kQK8_0);
            dst[0] = reinterpret_cast<uint4*>(q)[0];
            dst[1] = reinterpret_cast<uint4*>(q)[1];
        } else {
            __half h[32];
#pragma unroll
            for (int j = 0; j < 32; j++) h[j] = __int2half_rn((int)(int8_t)blk[2 + j]);
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(wq) + r * inner + b * kQK8_0);
#pragma unroll
            for (int j = 0; j < 4; j++) dst[j] = reinterpret_cast<uint4*>(h)[j];
        }
        if (kind == 2 || kind == 4) {
            __half g[16];
#pragma unroll
            for (int j = 0; j < 16; j++) g[j] = __ushort_as_half((unsigned short)0);
            g[b % 16] = __ushort_as_half((unsigned short)((uint16_t)blk[0] | ((uint16_t)blk[1] << 8)));
            uint4* gd = reinterpret_cast<uint4*>(ws1h + (r * nb + b) * 16);
            gd[0] = reinterpret_cast<uint4*>(g)[0];
            gd[1] = reinterpret_cast<uint4*>(g)[1];
        } else {
            dT[b * ldn + r] = load_half(blk);
        }
    }
}

__global__ void k_repack_q5_K(const uint8_t* __restrict__ raw, int64_t rows, int64_t inner, int64_t stride,
                              __half* __restrict__ wv, float* __restrict__ dT, float* __restrict__ dminT,
                              __half* __restrict__ bmin, int64_t ldn, int64_t gate_rows)
{
    const int64_t nsb = inner / kQKK;
    const int64_t total = rows * nsb * 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int g = (int)(i % 8);
        const int64_t sbi = i / 8;
        const int64_t r = sbi / nsb, sb = sbi % nsb;
        const uint8_t* blk = raw + src_row(r, gate_rows) * stride + sb * kQ5KBytes;
        int sc, mn;
        k_scale_min(blk + 4, g, sc, mn);
        const uint8_t* qh = blk + 16;
        const uint8_t* qs = blk + 48 + 32 * (g / 2);
        __half h[32];
#pragma unroll
        for (int t = 0; t < 32; t++) {
            int q = (g & 1) ? (qs[t] >> 4) : (qs[t] & 15);
            q += ((qh[t] >> g) & 1) << 4;
            h[t] = __int2half_rn(sc * q);
        }
        uint4* dst = reinterpret_cast<uint4*>(wv + r * inner + sb * kQKK + g * 32);
#pragma unroll
        for (int j = 0; j < 4; j++) dst[j] = reinterpret_cast<uint4*>(h)[j];
        __half2 pair = __halves2half2(__int2half_rn(64 * mn), __int2half_rn(mn));
        *reinterpret_cast<__half2*>(bmin + r * (nsb * 16) + sb * 16 + 2 * g) = pair;
        if (g == 0) {
            dT[sb * ldn + r] = load_half(blk);
            dminT[sb * ldn + r] = load_half(blk + 2);
        }
    }
}

// Q6_K rows as stored on the device: 224-byte padded super-blocks with the
// GGUF field offsets (ql at 0, qh at 128, scales at 192, d at 208).
__global__ void k_repack_q6_K(const uint8_t* __restrict__ raw, int64_t rows, int64_t inner, int64_t stride,
                              __half* __restrict__ wab, float* __restrict__ dT, int64_t ldn, int64_t gate_rows)
{
    const int64_t nsb = inner / kQKK;
    const int64_t total = rows * nsb * 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int G = (int)(i % 8);  // values 32G .. 32G+31 of the super-block
        const int64_t sbi = i / 8;
        const int64_t r = sbi / nsb, sb = sbi % nsb;
        const uint8_t* blk = raw + src_row(r, gate_rows) * stride + sb * kQ6KPadBytes;
        const int h = G / 4, g = G % 4;
        const uint8_t* ql = blk + 64 * h + 32 * (g % 2);
        const uint8_t* qh = blk + 128 + 32 * h;
        __half a[32], b[32];
#pragma unroll
        for (int t = 0; t < 32; t++) {
            int q = g < 2 ? (ql[t] & 15) : (ql[t] >> 4);
            q |= ((qh[t] >> (2 * g)) & 3) << 4;
            const int v = (int)(int8_t)blk[192 + 8 * h + 2 * g + t / 16] * (q - 32);
            a[t] = __int2half_rn(v & ~1);
            b[t] = __int2half_rn(v & 1);
        }
        const int64_t col = (sb * 4 + G / 2) * 128 + (G % 2) * 32;  // chunk G/2 of this super-block
        uint4* da = reinterpret_cast<uint4*>(wab + r * 2 * inner + col);
        uint4* db = reinterpret_cast<uint4*>(wab + r * 2 * inner + col + 64);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            da[j] = reinterpret_cast<uint4*>(a)[j];
            db[j] = reinterpret_cast<uint4*>(b)[j];
        }
        if (G == 0) dT[sb * ldn + r] = load_half(blk + 208);
    }
}

__global__ void k_decode(const uint8_t* __restrict__ data, uint32_t type, int64_t count, float* __restrict__ out)
{
    const int64_t blk_elems = type == kTypeQ8_0 ? kQK8_0 : kQKK;
    const int64_t total = count;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / blk_elems;
        const int e = (int)(i % blk_elems);
        if (type == kTypeQ8_0) {
            const uint8_t* blk = data + b * kQ8_0Bytes;
            out[i] = __fmul_rn((float)(int8_t)blk[2 + e], load_half(blk));
        } else if (type == kTypeQ5_K) {
            const uint8_t* blk = data + b * kQ5KBytes;
            const int g = e / 32, t = e % 32;
            int sc, mn;
            k_scale_min(blk + 4, g, sc, mn);
            int q = blk[48 + (g / 2) * 32 + t];
            q = (g & 1) ? (q >> 4) : (q & 15);
            if (blk[16 + t] & (1 << g)) q += 16;
            const float delta = load_half(blk), minimum = load_half(blk + 2);
            out[i] = __fsub_rn(__fmul_rn(__fmul_rn(delta, (float)sc), (float)q), __fmul_rn(minimum, (float)mn));
        } else {  // Q6_K
            const uint8_t* blk = data + b * kQ6KBytes;
            const int half = e / 128, g = (e % 128) / 32, t = e % 32;
            unsigned q = blk[half * 64 + t + (g % 2) * 32];
            q = g < 2 ? (q & 15u) : (q >> 4);
            q |= ((blk[128 + half * 32 + t] >> (g * 2)) & 3u) << 4;
            const float delta = load_half(blk + 208);
            const int8_t s = (int8_t)blk[192 + half * 8 + t / 16 + g * 2];
            out[i] = __fmul_rn(__fmul_rn(delta, (float)s), (float)((int)q - 32));
        }
    }
}

int grid_for(int64_t work, int threads)
{
    int64_t b = (work + threads - 1) / threads;
    if (b < 1) b = 1;
    if (b > 148 * 32) b = 148 * 32;
    return (int)b;
}

}  // namespace

cudaError_t launch_repack_q8_0(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, void* wq, float* dT,
                               __half* ws1h, int64_t ldn, int kind, int64_t gate_rows, cudaStream_t s)
{
    k_repack_q8_0<<<grid_for(rows * (inner / kQK8_0), 256), 256, 0, s>>>(raw, rows, inner, stride, wq, dT, ws1h, ldn, kind,
                                                                          gate_rows);
    return cudaGetLastError();
}

cudaError_t launch_repack_q5_K(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, __half* wv, float* dT,
                               float* dminT, __half* bmin, int64_t ldn, int64_t gate_rows, cudaStream_t s)
{
    k_repack_q5_K<<<grid_for(rows * (inner / kQKK) * 8, 256), 256, 0, s>>>(raw, rows, inner, stride, wv, dT, dminT, bmin, ldn,
                                                                         gate_rows);
    return cudaGetLastError();
}

cudaError_t launch_repack_q6_K(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, __half* wab, float* dT,
                               int64_t ldn, int64_t gate_rows, cudaStream_t s)
{
    k_repack_q6_K<<<grid_for(rows * (inner / kQKK) * 8, 256), 256, 0, s>>>(raw, rows, inner, stride, wab, dT, ldn, gate_rows);
    return cudaGetLastError();
}

cudaError_t launch_decode(const uint8_t* data, uint32_t type, int64_t count, float* out, cudaStream_t s)
{
    k_decode<<<grid_for(count, 256), 256, 0, s>>>(data, type, count, out);
    return cudaGetLastError();
}

}  // namespace pxq
