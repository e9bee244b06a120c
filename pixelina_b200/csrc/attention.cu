// attention.cu -- multi-head softmax attention in fp32, the callers' step
// after the quantized linears (tensor_attention, src/tensor.cpp:347-427).
//
// Semantics of the reference (both overloads): for query row t, head h and
// its key/value head kh = h / (heads / kv_heads), over the permitted key
// prefix j < L(t):  s_j = (q . k_j) / sqrt(d),  p_j = exp(s_j - max) / sum,
// out = sum_j p_j v_j.  L(t) comes from the query range holding t: key_end,
// or min(key_end, query_offset + t + 1) when the range is causal.  Layouts are
// the reference's row-major PixTensors: q and out [rows][heads*d], k and v
// [keys][kv_heads*d].  Everything is fp32 on the CUDA cores (the reference's
// arithmetic, not a reduced-precision tensor-core variant); the softmax is
// taken online over key tiles, which reorders the reference's sums (fp32
// rounding differences only).
//
//   k_attn         16-64 rows per CTA against 64-key tiles staged in shared
//                  memory, online softmax per row.  Prefill: a CTA takes one
//                  head and up to 64 query rows over all keys.  Decode (at
//                  most 8 query rows): a CTA takes every head of one
//                  key/value head (up to 64 head x row pairs, so each key and
//                  value is read once for the whole group) over one key
//                  split and writes partial (max, sum, out) per row;
//                  k_attn_combine merges the splits.
#include <cfloat>
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int KT = 64, ATT_THREADS = 256;
constexpr int64_t kSplitRows = 8;  // query rows up to which the keys are split across CTAs

struct AttnArgs {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    int64_t range_end[kAttnMaxRanges];   // query_end of each range (ascending)
    int64_t range_keys[kAttnMaxRanges];  // key_end
    int range_causal[kAttnMaxRanges];
    int nranges;
    int64_t q_rows, k_rows, query_offset;
    int heads, kv_heads;
    float scale;
    int vec;  // q, k, v and out are 16-byte aligned: whole float4 accesses
};

// Permitted key count of query row t.
__device__ __forceinline__ int64_t keys_of(const AttnArgs& a, int64_t t)
{
    int r = 0;
    while (r + 1 < a.nranges && t >= a.range_end[r]) r++;
    const int64_t ke = a.range_keys[r];
    if (!a.range_causal[r]) return ke;
    const int64_t c = a.query_offset + t + 1;
    return c < ke ? c : ke;
}

__device__ __forceinline__ float4 ld4(const float* p, bool vec)
{
    if (vec) return *reinterpret_cast<const float4*>(p);
    return make_float4(p[0], p[1], p[2], p[3]);
}

__device__ __forceinline__ void st4(float* p, float4 v, bool vec)
{
    if (vec) {
        *reinterpret_cast<float4*>(p) = v;
    } else {
        p[0] = v.x;
        p[1] = v.y;
        p[2] = v.z;
        p[3] = v.w;
    }
}

// 16-byte asynchronous copy global -> shared (zero fill when !valid; src is
// then not read), completion tracked per thread by commit/wait groups.
__device__ __forceinline__ void cp16(float* dst, const float* src, bool valid)
{
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_wait_prior() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// One CTA: QR = 16*RE rows against key tiles of KT keys.  A row is a (head,
// query row) pair: without SPLIT the CTA takes one head and QR consecutive
// query rows over all keys and writes the normalised output; with SPLIT it
// takes heads [hb, he) of one key/value head (all q_rows <= 8 rows of each)
// over one key range and writes partials (max pm, sum pl, unnormalised po)
// for k_attn_combine.  Queries and keys sit row-major in shared memory with
// stride D+4, so that the 4-word reads of thread tx (keys tx, tx+16, tx+32,
// tx+48) fall in distinct banks; a thread's block is RE rows (ty + 16f) x 4
// keys for the scores and RE rows x up to 8 output columns (float4 groups
// tx + 16h) for the values.  After the scores, the key buffer holds the
// tile's probabilities.  SPLIT CTAs (one per SM) double-buffer the key and
// value tiles: the copy of tile i+1 (cp.async, or plain loads when a tensor is
// not 16-byte aligned) runs while tile i is computed.  Prefill CTAs (two per
// SM, the other CTA hiding the copy) stage one tile at a time and write the
// probabilities over the keys once the scores are taken.
template <int D, int RE, bool SPLIT>
constexpr size_t attn_smem_bytes()
{
    constexpr int DP = D + 4, PS = KT + 4, QR = 16 * RE;
    return (size_t)(SPLIT ? QR * DP + 2 * KT * DP + 2 * KT * D + QR * PS : QR * DP + KT * DP + KT * D) * sizeof(float);
}

template <int D, int RE, bool SPLIT>
__global__ void __launch_bounds__(ATT_THREADS, SPLIT ? 1 : 2)
    k_attn(const __grid_constant__ AttnArgs a, int hpc, int hgroups, int64_t chunk, float* pm, float* pl, float* po)
{
    static_assert(D % 16 == 0 && D <= 128, "head size");
    constexpr bool PIPE = SPLIT;
    constexpr int DP = D + 4, PS = KT + 4, QR = 16 * RE, NG = D / 4, H = (NG + 15) / 16;
    static_assert(PIPE || QR * PS <= KT * DP, "probabilities fit over the keys");
    extern __shared__ float4 sm4[];
    float* qs = reinterpret_cast<float*>(sm4);          // [QR][DP] queries, pre-scaled
    float* kbuf = qs + QR * DP;                         // (2 x) [KT][DP] keys
    float* vbuf = kbuf + (PIPE ? 2 : 1) * KT * DP;      // (2 x) [KT][D]  values
    float* ps = PIPE ? vbuf + 2 * KT * D : kbuf;        // [QR][PS] the tile's probabilities
    __shared__ int64_t lim[QR];                 // permitted keys per row

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const bool vec = a.vec != 0;
    const int64_t qst = (int64_t)a.heads * D, kst = (int64_t)a.kv_heads * D;
    const int group = a.heads / a.kv_heads;
    int hb, he, kh;
    int64_t t0 = 0, kb = 0, ke = a.k_rows;
    if (SPLIT) {
        kh = blockIdx.x / hgroups;
        hb = kh * group + (int)(blockIdx.x % hgroups) * hpc;
        he = hb + hpc < (kh + 1) * group ? hb + hpc : (kh + 1) * group;
        kb = (int64_t)blockIdx.y * chunk;
        ke = kb + chunk < a.k_rows ? kb + chunk : a.k_rows;
    } else {
        hb = blockIdx.y;
        he = hb + 1;
        kh = hb / group;
        t0 = (int64_t)blockIdx.x * QR;
    }
    const int rows = (int)a.q_rows;
    // (head, query row) of CTA row lr; false past the CTA's rows
    auto row_of = [&](int lr, int& h, int64_t& t) -> bool {
        if (SPLIT) {
            h = hb + lr / rows;
            t = lr % rows;
            return h < he;
        }
        h = hb;
        t = t0 + lr;
        return t < a.q_rows;
    };

    for (int i = tid; i < QR * NG; i += ATT_THREADS) {
        const int lr = i / NG, g = i % NG;
        int h;
        int64_t t;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row_of(lr, h, t)) {
            x = ld4(a.q + t * qst + (int64_t)h * D + 4 * g, vec);
            x.x *= a.scale;
            x.y *= a.scale;
            x.z *= a.scale;
            x.w *= a.scale;
        }
        *reinterpret_cast<float4*>(qs + lr * DP + 4 * g) = x;
    }
    for (int lr = tid; lr < QR; lr += ATT_THREADS) {
        int h;
        int64_t t;
        lim[lr] = row_of(lr, h, t) ? keys_of(a, t) : 0;
    }
    __syncthreads();
    int64_t kmax = 0;
    for (int lr = 0; lr < QR; lr++) kmax = lim[lr] > kmax ? lim[lr] : kmax;
    if (ke > kmax) ke = kmax;  // keys past every row's limit contribute nothing

    float m[RE], l[RE], o[RE][H][4];
#pragma unroll
    for (int f = 0; f < RE; f++) {
        m[f] = -FLT_MAX;
        l[f] = 0.f;
#pragma unroll
        for (int hh = 0; hh < H; hh++)
#pragma unroll
            for (int c = 0; c < 4; c++) o[f][hh][c] = 0.f;
    }
    // copy the keys and values of tile [j0, j0 + KT) into buffer b
    auto stage = [&](int b, int64_t j0) {
        const int n = (int)(ke - j0 < KT ? ke - j0 : KT);
        float* kd = kbuf + b * KT * DP;
        float* vd = vbuf + b * KT * D;
        for (int i = tid; i < KT * NG; i += ATT_THREADS) {
            const int j = i / NG, g = i % NG;
            const int64_t off = (j0 + j) * kst + (int64_t)kh * D + 4 * g;
            if (PIPE && vec) {
                cp16(kd + j * DP + 4 * g, j < n ? a.k + off : a.k, j < n);
                cp16(vd + j * D + 4 * g, j < n ? a.v + off : a.v, j < n);
            } else {
                float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
                if (j < n) {
                    kv = ld4(a.k + off, vec);
                    vv = ld4(a.v + off, vec);
                }
                *reinterpret_cast<float4*>(kd + j * DP + 4 * g) = kv;
                *reinterpret_cast<float4*>(vd + j * D + 4 * g) = vv;
            }
        }
        if (PIPE) cp_commit();
    };
    if (PIPE && kb < ke) stage(0, kb);
    int cur = 0;
    for (int64_t j0 = kb; j0 < ke; j0 += KT, cur ^= PIPE ? 1 : 0) {
        const int n = (int)(ke - j0 < KT ? ke - j0 : KT);
        if (PIPE) {
            if (j0 + KT < ke) {
                stage(cur ^ 1, j0 + KT);  // buffer cur^1 was released by the barrier closing the previous tile
            } else {
                cp_commit();  // an empty group keeps "all but the newest group" meaning this tile
            }
            cp_wait_prior();
        } else {
            stage(0, j0);  // the barrier closing the previous tile released the buffers
        }
        __syncthreads();
        const float* ks = kbuf + cur * KT * DP;
        const float* vs = vbuf + cur * KT * D;
        float s[RE][4];
#pragma unroll
        for (int f = 0; f < RE; f++)
#pragma unroll
            for (int e = 0; e < 4; e++) s[f][e] = 0.f;
#pragma unroll 4
        for (int c = 0; c < D; c += 4) {
            float4 kf[4], qf[RE];
#pragma unroll
            for (int e = 0; e < 4; e++) kf[e] = *reinterpret_cast<const float4*>(ks + (tx + 16 * e) * DP + c);
#pragma unroll
            for (int f = 0; f < RE; f++) qf[f] = *reinterpret_cast<const float4*>(qs + (ty + 16 * f) * DP + c);
#pragma unroll
            for (int f = 0; f < RE; f++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float acc = s[f][e];
                    acc = __fmaf_rn(qf[f].x, kf[e].x, acc);
                    acc = __fmaf_rn(qf[f].y, kf[e].y, acc);
                    acc = __fmaf_rn(qf[f].z, kf[e].z, acc);
                    s[f][e] = __fmaf_rn(qf[f].w, kf[e].w, acc);
                }
        }
        if (!PIPE) __syncthreads();  // every thread is done with the keys: their buffer takes the probabilities
        // online softmax per row; the 16 threads of a half warp hold a row's 64 scores
#pragma unroll
        for (int f = 0; f < RE; f++) {
            const int lr = ty + 16 * f;
            const int64_t L = lim[lr];
            float tm = -FLT_MAX;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int j = tx + 16 * e;
                if (j >= n || j0 + j >= L) s[f][e] = -FLT_MAX;
                tm = fmaxf(tm, s[f][e]);
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
            const float mn = fmaxf(m[f], tm);
            float ts = 0.f;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float p = s[f][e] == -FLT_MAX ? 0.f : expf(s[f][e] - mn);
                ps[lr * PS + tx + 16 * e] = p;
                ts += p;
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) ts += __shfl_xor_sync(0xffffffffu, ts, off);
            const float corr = m[f] == -FLT_MAX ? 0.f : expf(m[f] - mn);
            l[f] = __fmaf_rn(l[f], corr, ts);
#pragma unroll
            for (int hh = 0; hh < H; hh++)
#pragma unroll
                for (int c = 0; c < 4; c++) o[f][hh][c] *= corr;
            m[f] = mn;
        }
        __syncthreads();
        const int nj = (n + 3) & ~3;  // probabilities past n are 0, value rows past n are zero
        for (int j = 0; j < nj; j += 4) {
            float4 pf[RE];
#pragma unroll
            for (int f = 0; f < RE; f++) pf[f] = *reinterpret_cast<const float4*>(ps + (ty + 16 * f) * PS + j);
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
#pragma unroll
                for (int hh = 0; hh < H; hh++) {
                    const int g = tx + 16 * hh;
                    if (NG % 16 != 0 && g >= NG) continue;
                    const float4 vv = *reinterpret_cast<const float4*>(vs + (j + jj) * D + 4 * g);
#pragma unroll
                    for (int f = 0; f < RE; f++) {
                        const float p = jj == 0 ? pf[f].x : jj == 1 ? pf[f].y : jj == 2 ? pf[f].z : pf[f].w;
                        o[f][hh][0] = __fmaf_rn(p, vv.x, o[f][hh][0]);
                        o[f][hh][1] = __fmaf_rn(p, vv.y, o[f][hh][1]);
                        o[f][hh][2] = __fmaf_rn(p, vv.z, o[f][hh][2]);
                        o[f][hh][3] = __fmaf_rn(p, vv.w, o[f][hh][3]);
                    }
                }
            }
        }
        __syncthreads();  // probabilities and buffer cur are consumed
    }
#pragma unroll
    for (int f = 0; f < RE; f++) {
        int h;
        int64_t t;
        if (!row_of(ty + 16 * f, h, t)) continue;
        if (SPLIT) {
            const int64_t part = ((int64_t)blockIdx.y * rows + t) * a.heads + h;
            if (tx == 0) {
                pm[part] = m[f];
                pl[part] = l[f];
            }
#pragma unroll
            for (int hh = 0; hh < H; hh++) {
                const int g = tx + 16 * hh;
                if (NG % 16 != 0 && g >= NG) continue;
                st4(po + part * D + 4 * g, make_float4(o[f][hh][0], o[f][hh][1], o[f][hh][2], o[f][hh][3]), true);
            }
        } else {
            const float inv = l[f] > 0.f ? 1.f / l[f] : 0.f;
            float* dst = a.out + t * qst + (int64_t)h * D;
#pragma unroll
            for (int hh = 0; hh < H; hh++) {
                const int g = tx + 16 * hh;
                if (NG % 16 != 0 && g >= NG) continue;
                st4(dst + 4 * g, make_float4(o[f][hh][0] * inv, o[f][hh][1] * inv, o[f][hh][2] * inv, o[f][hh][3] * inv),
                    vec);
            }
        }
    }
}

// Merge the key splits: out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.
// One CTA of 128 threads per (query row, head): the split weights first (a
// max and a sum over the CTA), then one output column per thread over the
// splits, loads unrolled so that several are in flight.
template <int D>
__global__ void __launch_bounds__(128) k_attn_combine(const __grid_constant__ AttnArgs a, int splits, const float* pm,
                                                      const float* pl, const float* po)
{
    extern __shared__ float wsplit[];  // [splits] weights e^(m_s - M)
    __shared__ float red[4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t rh = blockIdx.x;  // r * heads + h
    const int64_t stride = a.q_rows * a.heads;
    float mx = -FLT_MAX;
    for (int sp = tid; sp < splits; sp += 128) mx = fmaxf(mx, pm[sp * stride + rh]);
#pragma unroll
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float ls = 0.f;
    for (int sp = tid; sp < splits; sp += 128) {
        const float ms = pm[sp * stride + rh];
        const float w = ms == -FLT_MAX ? 0.f : expf(ms - M);
        wsplit[sp] = w;
        ls = __fmaf_rn(pl[sp * stride + rh], w, ls);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
    if (lane == 0) red[warp] = ls;
    __syncthreads();
    const float L = (red[0] + red[1]) + (red[2] + red[3]);
    if (tid >= D) return;
    float acc = 0.f;
    const float* col = po + rh * D + tid;
    int sp = 0;
    for (; sp + 8 <= splits; sp += 8) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) x[u] = col[(sp + u) * stride * D];
#pragma unroll
        for (int u = 0; u < 8; u++) acc = __fmaf_rn(x[u], wsplit[sp + u], acc);
    }
    for (; sp < splits; sp++) acc = __fmaf_rn(col[sp * stride * D], wsplit[sp], acc);
    const int64_t r = rh / a.heads, h = rh % a.heads;
    a.out[r * (int64_t)a.heads * D + h * D + tid] = L > 0.f ? acc / L : 0.f;
}

// Key-split plan of the decode path (q_rows <= kSplitRows): heads per CTA, CTAs
// per key/value head, keys per split (whole tiles) and the split count, sized
// for one CTA per SM.
struct SplitPlan {
    int hpc, hgroups;
    int64_t chunk, splits, parts;
};

SplitPlan plan_split(int64_t q_rows, int heads, int kv_heads, int64_t k_rows, int num_sms)
{
    SplitPlan p{};
    const int group = heads / kv_heads;
    p.hpc = (int)(64 / q_rows) < group ? (int)(64 / q_rows) : group;
    p.hgroups = (group + p.hpc - 1) / p.hpc;
    const int64_t base = (int64_t)kv_heads * p.hgroups;
    int64_t splits = ((int64_t)num_sms + base - 1) / base;
    const int64_t tiles = (k_rows + KT - 1) / KT;
    if (splits > tiles) splits = tiles;
    if (splits < 1) splits = 1;
    p.chunk = (tiles + splits - 1) / splits * KT;
    p.splits = (k_rows + p.chunk - 1) / p.chunk;
    if (p.splits < 1) p.splits = 1;
    p.parts = p.splits * q_rows * heads;
    return p;
}

size_t split_scratch_bytes(const SplitPlan& p, int64_t head_dim)
{
    return ((size_t)(2 * p.parts + 3) / 4 * 4 + (size_t)p.parts * head_dim) * sizeof(float);
}

template <int D, int RE, bool SPLIT>
cudaError_t launch_tiles(const AttnArgs& a, dim3 grid, int hpc, int hgroups, int64_t chunk, float* pm, float* pl, float* po,
                         cudaStream_t s)
{
    constexpr size_t smem = attn_smem_bytes<D, RE, SPLIT>();
    cudaError_t e = cudaFuncSetAttribute(k_attn<D, RE, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_attn<D, RE, SPLIT><<<grid, ATT_THREADS, smem, s>>>(a, hpc, hgroups, chunk, pm, pl, po);
    return cudaGetLastError();
}

template <int D, bool SPLIT>
cudaError_t launch_rows(const AttnArgs& a, int64_t cta_rows, dim3 grid, int hpc, int hgroups, int64_t chunk, float* pm, float* pl,
                        float* po, cudaStream_t s)
{
    if (cta_rows <= 16) return launch_tiles<D, 1, SPLIT>(a, grid, hpc, hgroups, chunk, pm, pl, po, s);
    if (cta_rows <= 32) return launch_tiles<D, 2, SPLIT>(a, grid, hpc, hgroups, chunk, pm, pl, po, s);
    return launch_tiles<D, 4, SPLIT>(a, grid, hpc, hgroups, chunk, pm, pl, po, s);
}

template <int D>
cudaError_t launch_attention_d(const AttnArgs& a, float* scratch, size_t scratch_bytes, int num_sms, cudaStream_t s)
{
    if (a.q_rows <= kSplitRows) {
        const SplitPlan p = plan_split(a.q_rows, a.heads, a.kv_heads, a.k_rows, num_sms);
        if (split_scratch_bytes(p, D) > scratch_bytes) return cudaErrorInvalidValue;
        float* pm = scratch;
        float* pl = pm + p.parts;
        float* po = scratch + (2 * p.parts + 3) / 4 * 4;
        const dim3 grid((unsigned)(a.kv_heads * p.hgroups), (unsigned)p.splits);
        cudaError_t e = launch_rows<D, true>(a, (int64_t)p.hpc * a.q_rows, grid, p.hpc, p.hgroups, p.chunk, pm, pl, po, s);
        if (e != cudaSuccess) return e;
        const size_t wbytes = (size_t)p.splits * sizeof(float);
        if (wbytes > 48 * 1024) return cudaErrorInvalidValue;
        k_attn_combine<D><<<(unsigned)(a.q_rows * a.heads), 128, wbytes, s>>>(a, (int)p.splits, pm, pl, po);
        return cudaGetLastError();
    }
    const int64_t cta_rows = a.q_rows <= 16 ? 16 : a.q_rows <= 32 ? 32 : 64;
    const dim3 grid((unsigned)((a.q_rows + cta_rows - 1) / cta_rows), (unsigned)a.heads);
    return launch_rows<D, false>(a, cta_rows, grid, 1, 1, 0, nullptr, nullptr, nullptr, s);
}

}  // namespace

size_t attention_scratch_bytes(int64_t q_rows, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t k_rows, int num_sms)
{
    if (q_rows > kSplitRows) return 0;
    return split_scratch_bytes(plan_split(q_rows, (int)heads, (int)kv_heads, k_rows, num_sms), head_dim);
}

cudaError_t launch_attention(const float* q, int64_t q_rows, const float* k, const float* v, int64_t k_rows, int heads,
                             int kv_heads, int head_dim, const int64_t* range_end, const int64_t* range_keys,
                             const int* range_causal, int nranges, int64_t query_offset, float* out, float* scratch,
                             size_t scratch_bytes, int num_sms, cudaStream_t s)
{
    if (nranges < 1 || nranges > kAttnMaxRanges) return cudaErrorInvalidValue;
    AttnArgs a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    for (int i = 0; i < nranges; i++) {
        a.range_end[i] = range_end[i];
        a.range_keys[i] = range_keys[i];
        a.range_causal[i] = range_causal[i];
    }
    a.nranges = nranges;
    a.q_rows = q_rows;
    a.k_rows = k_rows;
    a.query_offset = query_offset;
    a.heads = heads;
    a.kv_heads = kv_heads;
    a.scale = 1.0f / sqrtf((float)head_dim);
    a.vec = (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) == 0;
    switch (head_dim) {
    case 64: return launch_attention_d<64>(a, scratch, scratch_bytes, num_sms, s);
    case 80: return launch_attention_d<80>(a, scratch, scratch_bytes, num_sms, s);
    case 128: return launch_attention_d<128>(a, scratch, scratch_bytes, num_sms, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace pxq
