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
//   k_attn_tiled   64 query rows x one head per CTA, 64-key tiles staged in
//                  shared memory (keys and queries transposed so that a
//                  thread's 4x4 score block and 4x(d/16) output block read
//                  whole float4 words), online softmax per row.
//   k_attn_split   few query rows (decode): one CTA per (head, key split),
//                  partial (max, sum, out) per query row; k_attn_combine
//                  merges the splits.
#include <cfloat>
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int BQ = 64, BKT = 64, ATT_THREADS = 256;

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

template <int D>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_tiled(const __grid_constant__ AttnArgs a)
{
    static_assert(D % 16 == 0 && D <= 128, "head size");
    constexpr int OC = D / 16;  // output columns per thread
    extern __shared__ float sm[];
    float* qt = sm;                 // [D][BQ]   queries, transposed
    float* kt = qt + D * BQ;        // [D][BKT]  keys, transposed
    float* vs = kt + D * BKT;       // [BKT][D]  values
    float* ps = vs + BKT * D;       // [BQ][BKT] probabilities of the tile
    __shared__ int64_t lim[BQ];     // permitted keys per query row

    const int h = blockIdx.y, kh = h / (a.heads / a.kv_heads);
    const int64_t t0 = (int64_t)blockIdx.x * BQ;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;  // 16 x 16 threads
    const int64_t qs = (int64_t)a.heads * D, ks = (int64_t)a.kv_heads * D;

    for (int i = tid; i < BQ * D; i += ATT_THREADS) {
        const int r = i / D, c = i % D;
        const int64_t t = t0 + r;
        qt[c * BQ + r] = t < a.q_rows ? a.q[t * qs + (int64_t)h * D + c] * a.scale : 0.f;
    }
    int64_t kmax = 0;
    for (int r = tid; r < BQ; r += ATT_THREADS) lim[r] = t0 + r < a.q_rows ? keys_of(a, t0 + r) : 0;
    __syncthreads();
    for (int r = 0; r < BQ; r++) kmax = lim[r] > kmax ? lim[r] : kmax;

    // rows ty*4 .. ty*4+3; score columns tx*4 .. tx*4+3; output columns tx*OC .. tx*OC+OC-1
    float m[4], l[4], o[4][OC];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -FLT_MAX;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < OC; c++) o[i][c] = 0.f;
    }
    for (int64_t j0 = 0; j0 < kmax; j0 += BKT) {
        __syncthreads();  // the previous tile's keys, values and probabilities are consumed
        for (int i = tid; i < BKT * D; i += ATT_THREADS) {
            const int j = i / D, c = i % D;
            const int64_t key = j0 + j;
            const bool in = key < a.k_rows;
            kt[c * BKT + j] = in ? a.k[key * ks + (int64_t)kh * D + c] : 0.f;
            vs[j * D + c] = in ? a.v[key * ks + (int64_t)kh * D + c] : 0.f;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = 0.f;
#pragma unroll 8
        for (int c = 0; c < D; c++) {
            const float4 qv = *reinterpret_cast<const float4*>(qt + c * BQ + ty * 4);
            const float4 kv = *reinterpret_cast<const float4*>(kt + c * BKT + tx * 4);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = __fmaf_rn(qa[i], ka[j], s[i][j]);
        }
        // online softmax over this tile, per row (16 threads of a half warp share a row group)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int64_t L = lim[ty * 4 + i];
            float tm = -FLT_MAX;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (j0 + tx * 4 + j >= L) s[i][j] = -FLT_MAX;
                tm = fmaxf(tm, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
            const float mn = fmaxf(m[i], tm);
            float ts = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float e = s[i][j] == -FLT_MAX ? 0.f : expf(s[i][j] - mn);
                ps[(ty * 4 + i) * BKT + tx * 4 + j] = e;
                ts += e;
            }
#pragma unroll
            for (int off = 8; off; off >>= 1) ts += __shfl_xor_sync(0xffffffffu, ts, off);
            const float corr = m[i] == -FLT_MAX ? 0.f : expf(m[i] - mn);
            l[i] = __fmaf_rn(l[i], corr, ts);
#pragma unroll
            for (int c = 0; c < OC; c++) o[i][c] *= corr;
            m[i] = mn;
        }
        __syncthreads();
        const int64_t jn = kmax - j0 < BKT ? kmax - j0 : BKT;
        for (int j = 0; j < jn; j++) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; i++) p[i] = ps[(ty * 4 + i) * BKT + j];
            const float* vr = vs + j * D + tx * OC;
#pragma unroll
            for (int c = 0; c < OC; c++) {
                const float vv = vr[c];
#pragma unroll
                for (int i = 0; i < 4; i++) o[i][c] = __fmaf_rn(p[i], vv, o[i][c]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int64_t t = t0 + ty * 4 + i;
        if (t >= a.q_rows) continue;
        const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
        float* dst = a.out + t * qs + (int64_t)h * D + tx * OC;
#pragma unroll
        for (int c = 0; c < OC; c++) dst[c] = o[i][c] * inv;
    }
}

// Decode: CTA (head h, split sp) over keys [sp*chunk, (sp+1)*chunk) for every
// query row (at most 8).  Partials per (split, row, head): running max pm,
// sum pl, unnormalised output po[D].
template <int D>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_split(const __grid_constant__ AttnArgs a, int64_t chunk, float* pm, float* pl,
                                                            float* po)
{
    constexpr int R = 8, SUB = 256, KW = (D + 31) / 32;
    constexpr int RSTEP = ATT_THREADS / D;  // output rows covered per pass
    __shared__ float qv[R][D];
    __shared__ float sc[R][SUB];
    __shared__ float corr[R], mrow[R], lrow[R];
    __shared__ int64_t lim[R];
    const int h = blockIdx.x, kh = h / (a.heads / a.kv_heads), sp = blockIdx.y;
    const int rows = (int)a.q_rows;
    const int64_t qs = (int64_t)a.heads * D, ks = (int64_t)a.kv_heads * D;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < R * D; i += ATT_THREADS) {
        const int r = i / D, c = i % D;
        qv[r][c] = r < rows ? a.q[(int64_t)r * qs + (int64_t)h * D + c] * a.scale : 0.f;
    }
    if (tid < R) {
        lim[tid] = tid < rows ? keys_of(a, tid) : 0;
        mrow[tid] = -FLT_MAX;
        lrow[tid] = 0.f;
    }
    // thread tid < RSTEP*D owns column tid % D of rows tid / D + RSTEP*u
    const bool owner = tid < RSTEP * D;
    const int oc = tid % D, orow = tid / D;
    float o[(R + RSTEP - 1) / RSTEP];
#pragma unroll
    for (int u = 0; u < (R + RSTEP - 1) / RSTEP; u++) o[u] = 0.f;
    const int64_t k0 = (int64_t)sp * chunk;
    const int64_t k1 = k0 + chunk < a.k_rows ? k0 + chunk : a.k_rows;
    for (int64_t j0 = k0; j0 < k1; j0 += SUB) {
        const int n = (int)(k1 - j0 < SUB ? k1 - j0 : SUB);
        __syncthreads();  // q and the row state are written; the previous sub-chunk's probabilities are consumed
        for (int j = warp; j < n; j += ATT_THREADS / 32) {
            const float* kr = a.k + (j0 + j) * ks + (int64_t)kh * D;
            float kk[KW];
#pragma unroll
            for (int u = 0; u < KW; u++) kk[u] = lane + 32 * u < D ? kr[lane + 32 * u] : 0.f;
            for (int r = 0; r < rows; r++) {
                float acc = 0.f;
#pragma unroll
                for (int u = 0; u < KW; u++)
                    if (lane + 32 * u < D) acc = __fmaf_rn(qv[r][lane + 32 * u], kk[u], acc);
#pragma unroll
                for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
                if (lane == 0) sc[r][j] = j0 + j < lim[r] ? acc : -FLT_MAX;
            }
        }
        __syncthreads();
        if (warp < rows) {  // warp r: row r's new max, probabilities, sum, rescale factor
            const int r = warp;
            float tm = -FLT_MAX;
            for (int j = lane; j < n; j += 32) tm = fmaxf(tm, sc[r][j]);
#pragma unroll
            for (int off = 16; off; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
            const float mo = mrow[r], mn = fmaxf(mo, tm);
            float ts = 0.f;
            for (int j = lane; j < n; j += 32) {
                const float e = sc[r][j] == -FLT_MAX ? 0.f : expf(sc[r][j] - mn);
                sc[r][j] = e;
                ts += e;
            }
#pragma unroll
            for (int off = 16; off; off >>= 1) ts += __shfl_xor_sync(0xffffffffu, ts, off);
            if (lane == 0) {
                const float cf = mo == -FLT_MAX ? 0.f : expf(mo - mn);
                corr[r] = cf;
                lrow[r] = __fmaf_rn(lrow[r], cf, ts);
                mrow[r] = mn;
            }
        }
        __syncthreads();
        if (owner) {
#pragma unroll
            for (int u = 0; u < (R + RSTEP - 1) / RSTEP; u++) {
                const int r = orow + RSTEP * u;
                if (r < rows) o[u] *= corr[r];
            }
            for (int j = 0; j < n; j++) {
                const float vv = a.v[(j0 + j) * ks + (int64_t)kh * D + oc];
#pragma unroll
                for (int u = 0; u < (R + RSTEP - 1) / RSTEP; u++) {
                    const int r = orow + RSTEP * u;
                    if (r < rows) o[u] = __fmaf_rn(sc[r][j], vv, o[u]);
                }
            }
        }
    }
    __syncthreads();
    const int64_t base = ((int64_t)sp * rows) * a.heads;
    if (tid < rows) {
        pm[base + (int64_t)tid * a.heads + h] = mrow[tid];
        pl[base + (int64_t)tid * a.heads + h] = lrow[tid];
    }
    if (owner) {
#pragma unroll
        for (int u = 0; u < (R + RSTEP - 1) / RSTEP; u++) {
            const int r = orow + RSTEP * u;
            if (r < rows) po[(base + (int64_t)r * a.heads + h) * D + oc] = o[u];
        }
    }
}

// Merge the key splits: out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s.
template <int D>
__global__ void k_attn_combine(const __grid_constant__ AttnArgs a, int splits, const float* pm, const float* pl, const float* po)
{
    const int rows = (int)a.q_rows;
    const int64_t total = (int64_t)rows * a.heads * D;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % D);
        const int64_t rh = i / D;  // r * heads + h
        float M = -FLT_MAX;
        for (int s = 0; s < splits; s++) M = fmaxf(M, pm[(int64_t)s * rows * a.heads + rh]);
        float L = 0.f, acc = 0.f;
        for (int s = 0; s < splits; s++) {
            const float ms = pm[(int64_t)s * rows * a.heads + rh];
            if (ms == -FLT_MAX) continue;
            const float w = expf(ms - M);
            L = __fmaf_rn(pl[(int64_t)s * rows * a.heads + rh], w, L);
            acc = __fmaf_rn(po[((int64_t)s * rows * a.heads + rh) * D + c], w, acc);
        }
        const int64_t r = rh / a.heads, h = rh % a.heads;
        a.out[r * (int64_t)a.heads * D + h * D + c] = L > 0.f ? acc / L : 0.f;
    }
}

template <int D>
cudaError_t launch_attention_d(const AttnArgs& a, float* scratch, size_t scratch_bytes, int num_sms, cudaStream_t s)
{
    if (a.q_rows <= 8) {
        // split the keys so that about two CTAs per SM work
        int64_t splits = (2 * (int64_t)num_sms + a.heads - 1) / a.heads;
        const int64_t max_splits = (a.k_rows + 63) / 64;
        if (splits > max_splits) splits = max_splits;
        if (splits < 1) splits = 1;
        const int64_t chunk = (a.k_rows + splits - 1) / splits;
        splits = (a.k_rows + chunk - 1) / chunk;
        const int64_t parts = splits * a.q_rows * a.heads;
        if ((size_t)parts * (2 + D) * sizeof(float) > scratch_bytes) return cudaErrorInvalidValue;
        float* pm = scratch;
        float* pl = pm + parts;
        float* po = pl + parts;
        k_attn_split<D><<<dim3((unsigned)a.heads, (unsigned)splits), ATT_THREADS, 0, s>>>(a, chunk, pm, pl, po);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        const int64_t total = a.q_rows * a.heads * D;
        int64_t blocks = (total + 255) / 256;
        if (blocks > 4 * num_sms) blocks = 4 * num_sms;
        k_attn_combine<D><<<(unsigned)blocks, 256, 0, s>>>(a, (int)splits, pm, pl, po);
        return cudaGetLastError();
    }
    constexpr size_t smem = (size_t)(D * BQ + D * BKT + BKT * D + BQ * BKT) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(k_attn_tiled<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((a.q_rows + BQ - 1) / BQ), (unsigned)a.heads);
    k_attn_tiled<D><<<grid, ATT_THREADS, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

size_t attention_scratch_bytes(int64_t q_rows, int64_t heads, int64_t head_dim, int num_sms)
{
    if (q_rows > 8) return 0;
    const int64_t splits = (2 * (int64_t)num_sms + heads - 1) / heads;
    return (size_t)splits * q_rows * heads * (2 + head_dim) * sizeof(float);
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
    switch (head_dim) {
    case 64: return launch_attention_d<64>(a, scratch, scratch_bytes, num_sms, s);
    case 80: return launch_attention_d<80>(a, scratch, scratch_bytes, num_sms, s);
    case 128: return launch_attention_d<128>(a, scratch, scratch_bytes, num_sms, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace pxq
