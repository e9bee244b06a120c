// matvec.cu -- small-M (decode) quantized matvec: y = X * W^T for M <= 8.
//
// Restates, for columns <= 8, the inner loop of cpu_quant_matmul
// (src/kernels_quant.cpp:389-400) with the dots pix_dot_q8_0 (:339-365) and
// pix_dot_q5_K (:163-254) on GPU: activations are quantized exactly as the
// reference quantizes them (quantize.cu), weights stream straight from the
// raw GGUF rows in HBM.  Every 32-value block dot is one int8 tensor-core
// mma.sync m16n8k32: A = 16 weight rows unpacked in registers, B = the up-to-8
// activation rows (n = activation row, zero-padded), so one weight fragment
// serves all rows.  The exact int32 block dot comes out of the MMA; the
// per-block fp32 scaling and the Q5_K sub-block scales / min term are applied
// exactly as the reference does (int32 super-block sums, then one fp32 FMA
// per super-block).  The K order inside a 32-block is permuted identically for
// A and B (a dot product does not depend on the order of its terms) so that
// each thread's 8 weight bytes per block are contiguous in memory.  All sums
// across warps, stages and CTAs are taken in a fixed order: results are
// deterministic.
//
// Q5_K (the decode format): a persistent, warp-specialised stream-K kernel.
// One producer warp streams 64-row x 2-super-block weight tiles (22.5 KB),
// and the matching activation records, into a 4-stage shared-memory ring with
// TMA / bulk copies; eight consumer warps (4 row groups x 2 super-block
// halves) unpack them into MMA fragments.  The stage sequence of all tiles is
// split evenly over one CTA per SM, so every SM streams the same number of
// bytes whatever the matrix shape; a tile shared by several CTAs is summed,
// in CTA order, by the last to finish.  Launched with programmatic stream
// serialization, and sized (110 KB of shared memory, 288 threads) so that a
// CTA of the next such kernel fits on the same SM: the producer requests its
// first stages' weights as soon as the CTA is resident, while the kernels
// before it still run, and waits for them (griddep_wait) before it fetches
// activations; the consumers wait before touching any output.
//
// Q8_0 runs in the same kernel when K is a multiple of 256: a "super-block"
// is then eight raw 34-byte blocks (272 bytes, so rows are 16-byte multiples
// as TMA needs), streamed by the same 3-D tensor maps; each block is one MMA
// whose quants the consumers read from shared memory with aligned loads and
// funnel shifts, and the activation records hold the blocks' quants in the
// fragment layout plus their scales as fp32.  Other K: a CTA of 4 warps owns
// 16 weight rows and a range of K blocks (the whole row, or a 1/ks slice when
// there are too few row groups to fill the GPU); warps walk the blocks
// round-robin with the next block's weight bytes in flight (register double
// buffering).
#include <atomic>

#include "pxq_device.cuh"
#include "pxq_internal.h"
#include "q8k.cuh"

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

// The same two loads for activation bytes, which the kernel before this one
// writes (coherent loads, see ld_dep_u32).
__device__ __forceinline__ uint2 ld8_unaligned_dep(const uint8_t* p)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    const uint32_t sh = (uint32_t)(a & 3u) * 8u;
    const uint32_t w0 = ld_dep_u32(w), w1 = ld_dep_u32(w + 1);
    const uint32_t w2 = sh ? ld_dep_u32(w + 2) : 0u;
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

__device__ __forceinline__ float ld_half_dep(const uint8_t* p)
{
    return __half2float(__ushort_as_half(ld_dep_u16(p)));
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
                                                          int64_t inner, const uint8_t* xq, int64_t columns,
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
    griddep_launch_dependents();
    if (b < b1) {
        if (va) { qa = ld8_unaligned(wa + b * kQ8_0Bytes + 2 + 8 * t); dwa = ld_half(wa + b * kQ8_0Bytes); }
        if (vb) { qb = ld8_unaligned(wb + b * kQ8_0Bytes + 2 + 8 * t); dwb = ld_half(wb + b * kQ8_0Bytes); }
    }
    // weights above are read-only; the activation, outputs and split-K
    // scratch belong to the kernels before this one
    griddep_wait();
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
        const uint2 qx = vx ? ld8_unaligned_dep(xr + off + 2 + 8 * t) : make_uint2(0, 0);
        const uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
        int d[4];
        mma_s8(d, a, qx.x, qx.y);
        const float dx0 = ld_half_dep(xc0 + off), dx1 = ld_half_dep(xc1 + off);
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

constexpr int kMvFusedRecords = 32;  // activation records a CTA may quantize itself (the plan checks)

__device__ __forceinline__ void mma_u8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0)
{
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Weight formats of the TMA-fed matvec: bytes of one 256-value super-block
// as stored on the device, the activation record it reads (quantize.cu,
// q8k.cuh), and whether 64-row stages land row-major (Q5_K: a 352-byte row
// pitch spreads the fragment loads over the banks; Q6_K's 448 would not).
template <uint32_t WT>
struct MvFmt;
template <>
struct MvFmt<kTypeQ5_K> {
    static constexpr int kSbBytes = kQ5KBytes;    // 176
    static constexpr int kRecBytes = kQ8KMvBytes; // 288
    static constexpr bool kRowMajor64 = true;
};
template <>
struct MvFmt<kTypeQ6_K> {
    static constexpr int kSbBytes = kQ6KPadBytes; // 224: 210 bytes padded at upload
    static constexpr int kRecBytes = kQ8KQ6Bytes; // 304
    static constexpr bool kRowMajor64 = false;
};
template <>
struct MvFmt<kTypeQ8_0> {
    static constexpr int kSbBytes = kQ80SbBytes;  // 272: eight raw 34-byte blocks
    static constexpr int kRecBytes = kQ80MvBytes; // 288
    static constexpr bool kRowMajor64 = false;
};

// Tile shapes: TR weight rows x 128/TR super-blocks per stage.  Every stage is
// 128 row-super-blocks of weights (22.5 KB of Q5_K, 28 KB of Q6_K); consumer
// warp w takes rows 16*(w % (TR/16)) .. +15 of the tile and super-block
// w / (TR/16) of the stage, so all eight warps work on every stage whatever
// the shape.  A Q5_K 64-row stage lands in shared memory row-major ([64][352
// B], a 2-D box); the others super-block-major ([sb][TR][sb bytes], a 3-D
// box), because a row pitch that is a multiple of 128 bytes would put all
// rows of a fragment load in the same banks.
template <int TR, bool FUSED, uint32_t WT>
struct MvShape {
    using Fmt = MvFmt<WT>;
    static constexpr bool kRowMajor = TR == 64 && Fmt::kRowMajor64;
    static constexpr int kRowGroups = TR / 16;                      // 16-row MMA groups per tile
    static constexpr int kSbs = kMvStageSuperBlocks / kRowGroups;    // super-blocks per stage
    static constexpr int kRowBytes = kSbs * Fmt::kSbBytes;          // one row's bytes per stage
    static constexpr int kRowPitch = kRowMajor ? kRowBytes : Fmt::kSbBytes;    // shared-memory row pitch
    static constexpr int kSbPitch = kRowMajor ? Fmt::kSbBytes : TR * Fmt::kSbBytes;  // super-block pitch
    static constexpr int kWeightBytes = TR * kRowBytes;
    static constexpr int kActPitch = kSbs * Fmt::kRecBytes;         // one activation row's records per stage
    static constexpr int kActBytes = 8 * kActPitch + 512;           // up to 8 activation rows, skewed
    // two CTAs per SM within 228 KB; with a fused quantize there is no
    // per-stage activation buffer, so the Q5_K weight ring gets a fourth
    // stage; Q8_0 stages are 34 KB, two of them
    static constexpr int kStages = WT == kTypeQ8_0 ? 2 : FUSED ? (WT == kTypeQ5_K ? 4 : 3) : (TR == 16 ? 2 : 3);
    static_assert(kRowBytes % 16 == 0 && kActPitch % 16 == 0, "bulk copies move 16-byte multiples");
    static_assert(kWeightBytes == 16 * kMvStageSuperBlocks * Fmt::kSbBytes, "every shape streams the same stage size");
};

constexpr int kMvConsumers = 8;
constexpr int kMvProducerWarp = kMvConsumers;            // TMA / bulk-copy issue
constexpr int kMvFixupWarp = kMvConsumers + 1;           // cross-CTA sums of shared tiles
constexpr int kMvThreads = (kMvConsumers + 2) * 32;

template <int TR, bool FUSED, uint32_t WT>
struct MvSmem {
    using Sh = MvShape<TR, FUSED, WT>;
    static constexpr int kRec = MvFmt<WT>::kRecBytes;
    // activation: per-stage buffers (8 rows of kSbs records at act_row_off),
    // or with a fused quantize the records of all of the CTA's stages plus
    // one zero record
    static constexpr int kActAreaBytes = FUSED ? (kMvFusedRecords + 1) * kRec : Sh::kStages * Sh::kActBytes;
    uint8_t weight[Sh::kStages][Sh::kWeightBytes];
    uint8_t act_area[kActAreaBytes];
    // sums of warps with super-block lane >= 1, handed to lane 0, by segment parity
    float red[2][Sh::kSbs - 1][Sh::kRowGroups][16][8];
    uint64_t full[Sh::kStages], empty[Sh::kStages];
    uint64_t part;                                   // the first shared tile's partial sums are stored
    uint32_t abort;
    uint32_t last;                                   // this CTA completes its last shared tile
    __device__ uint8_t* act(uint32_t k) { return act_area + k * Sh::kActBytes; }
};

struct MvParams {
    CUtensorMap map;                   // weight bytes: 2-D u64 [rows][stride/8], box {kRowBytes/8, TR} (row-major
                                       // stages), else 3-D u64 [nsb][rows][sb bytes/8], box {sb bytes/8, TR, kSbs}
    const uint8_t* act;                // activation records [columns][nsb][record bytes] (not fused)
    const float* x;                    // fp32 activation rows (fused quantize: the kernel's FUSED variant)
    int64_t ldx;
    float* y;
    const float* bias;
    float* partial;                    // [grid][2][columns][TR]
    uint32_t* counters;                // [tiles]
    uint32_t* status;
    int64_t ldy, rows, row_first, stages;
    int64_t gated_half;                // gated pair: F / 64; logical tile 2j = gate tile j, 2j+1 = up tile j
    int32_t nsb, spt, columns;
    int32_t stall;                     // testing: CTA 0 loads nothing (MatvecPlan::debug_stall)
};

// First CTA whose stage range [c*S/G, (c+1)*S/G) holds stage s.
__device__ __forceinline__ int64_t cta_of_stage(int64_t s, int64_t S, int64_t G) { return ((s + 1) * G - 1) / S; }

// Slot (0 or 1) of CTA c's partial sums for tile T: 0 for the first tile of
// its range, 1 for the last (only the first and last tiles can be partial).
__device__ __forceinline__ int64_t partial_slot(int64_t c, int64_t T, int64_t S, int64_t G, int64_t spt)
{
    return T == (c * S / G) / spt ? 0 : 1;
}

// Packed 6-bit scales and mins of one super-block header (bytes 4..15 as
// words h.y, h.z, h.w), four sub-blocks per word: sc[0..3], sc[4..7], m[0..3], m[4..7].
__device__ __forceinline__ void q5_scales(const uint4 h, uint32_t& sc_lo, uint32_t& sc_hi, uint32_t& mn_lo, uint32_t& mn_hi)
{
    sc_lo = h.y & 0x3f3f3f3fu;
    mn_lo = h.z & 0x3f3f3f3fu;
    sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
}

// Four 5-bit quants of sub-block J as int8 bytes: the low (E = 0) or high
// (E = 1) nibbles of q plus bit J of each byte of the high-bit word h.
template <int J, int E>
__device__ __forceinline__ uint32_t q5_frag(uint32_t q, uint32_t h)
{
    const uint32_t lo = (E ? (q >> 4) : q) & 0x0f0f0f0fu;
    const uint32_t hs = J <= 4 ? (h << (4 - J)) : (h >> (J - 4));
    return lo | (hs & 0x10101010u);
}

// sum_j m_j * bs_j over the 8 sub-blocks: bs = eight int16 32-element sums
// (two per word), m = eight 6-bit mins (four bytes per word).
__device__ __forceinline__ int min_dot(const uint4 bs, uint32_t m_lo, uint32_t m_hi)
{
    int r = __dp2a_lo((int)bs.x, (int)m_lo, 0);
    r = __dp2a_hi((int)bs.y, (int)m_lo, r);
    r = __dp2a_lo((int)bs.z, (int)m_hi, r);
    return __dp2a_hi((int)bs.w, (int)m_hi, r);
}

// Sub-blocks 2PR and 2PR+1 of one super-block for weight rows a, b (A) and
// activation row g (B); sca/scb hold the four packed scales of sub-blocks
// 4*(PR/2) .. 4*(PR/2)+3.  Every lane must call it: the MMA is warp-wide.
template <int PR>
__device__ __forceinline__ void q5_pair(const uint8_t* wa, const uint8_t* wb, const uint8_t* xr, uint32_t t, uint2 qha,
                                        uint2 qhb, uint32_t sca, uint32_t scb, int (&sumi)[4])
{
    // sub-blocks 2PR (low nibbles) and 2PR+1 (high nibbles) share these qs bytes
    const uint2 qa = *reinterpret_cast<const uint2*>(wa + 48 + 32 * PR + 8 * t);
    const uint2 qb = *reinterpret_cast<const uint2*>(wb + 48 + 32 * PR + 8 * t);
    const uint4 bx = *reinterpret_cast<const uint4*>(xr + 64 * PR);
    constexpr int kSh = 16 * (PR & 1);
    {
        constexpr int J = 2 * PR;
        const uint32_t a[4] = {q5_frag<J, 0>(qa.x, qha.x), q5_frag<J, 0>(qb.x, qhb.x), q5_frag<J, 0>(qa.y, qha.y),
                               q5_frag<J, 0>(qb.y, qhb.y)};
        int d[4];
        mma_s8(d, a, bx.x, bx.y);
        const int s0 = (int)((sca >> kSh) & 0xffu), s1 = (int)((scb >> kSh) & 0xffu);
        sumi[0] += s0 * d[0];
        sumi[1] += s0 * d[1];
        sumi[2] += s1 * d[2];
        sumi[3] += s1 * d[3];
    }
    {
        constexpr int J = 2 * PR + 1;
        const uint32_t a[4] = {q5_frag<J, 1>(qa.x, qha.x), q5_frag<J, 1>(qb.x, qhb.x), q5_frag<J, 1>(qa.y, qha.y),
                               q5_frag<J, 1>(qb.y, qhb.y)};
        int d[4];
        mma_s8(d, a, bx.z, bx.w);
        const int s0 = (int)((sca >> (kSh + 8)) & 0xffu), s1 = (int)((scb >> (kSh + 8)) & 0xffu);
        sumi[0] += s0 * d[0];
        sumi[1] += s0 * d[1];
        sumi[2] += s1 * d[2];
        sumi[3] += s1 * d[3];
    }
}

// One Q5_K super-block of weight rows a = g, b = g+8 against activation rows
// g (B fragments from record xg) and 2t, 2t+1 (32-element sums and scale
// from records x0, x1): the int32 super-block sums of pix_dot_q5_K, then its
// two fp32 FMAs.  Record layout: q8_K_store_mv (q8k.cuh).
__device__ __forceinline__ void q5_unit(const uint8_t* wa, const uint8_t* wb, const uint8_t* xg, const uint8_t* x0,
                                        const uint8_t* x1, uint32_t t, float (&acc)[4], float (&summ)[4])
{
    const uint4 ha = *reinterpret_cast<const uint4*>(wa), hb = *reinterpret_cast<const uint4*>(wb);
    const uint2 qha = *reinterpret_cast<const uint2*>(wa + 16 + 8 * t);
    const uint2 qhb = *reinterpret_cast<const uint2*>(wb + 16 + 8 * t);
    uint32_t sca_lo, sca_hi, mna_lo, mna_hi, scb_lo, scb_hi, mnb_lo, mnb_hi;
    q5_scales(ha, sca_lo, sca_hi, mna_lo, mna_hi);
    q5_scales(hb, scb_lo, scb_hi, mnb_lo, mnb_hi);
    const uint8_t* xr = xg + 16 * t;
    int sumi[4] = {0, 0, 0, 0};
    q5_pair<0>(wa, wb, xr, t, qha, qhb, sca_lo, scb_lo, sumi);
    q5_pair<1>(wa, wb, xr, t, qha, qhb, sca_lo, scb_lo, sumi);
    q5_pair<2>(wa, wb, xr, t, qha, qhb, sca_hi, scb_hi, sumi);
    q5_pair<3>(wa, wb, xr, t, qha, qhb, sca_hi, scb_hi, sumi);
    const uint4 s0 = *reinterpret_cast<const uint4*>(x0 + kQKK);
    const uint4 s1 = *reinterpret_cast<const uint4*>(x1 + kQKK);
    const int msum[4] = {min_dot(s0, mna_lo, mna_hi), min_dot(s1, mna_lo, mna_hi), min_dot(s0, mnb_lo, mnb_hi),
                         min_dot(s1, mnb_lo, mnb_hi)};
    const float dx0 = *reinterpret_cast<const float*>(x0 + kQKK + 16);
    const float dx1 = *reinterpret_cast<const float*>(x1 + kQKK + 16);
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

// Sign-extended byte k (0..15) of a 16-byte word group.
__device__ __forceinline__ int sbyte(const uint4 w, int k)
{
    const uint32_t v = k < 4 ? w.x : k < 8 ? w.y : k < 12 ? w.z : w.w;
    return (int)(int8_t)(uint8_t)(v >> (8 * (k & 3)));
}

// sum_s sc_s * bsum_s over the 16 sixteen-value groups: bs = 16 int16 sums
// (two per word), sc = 16 int8 scales (four per word).
__device__ __forceinline__ int q6_scaled_sums(const uint4 bs0, const uint4 bs1, const uint4 sc)
{
    int r = __dp2a_lo((int)bs0.x, (int)sc.x, 0);
    r = __dp2a_hi((int)bs0.y, (int)sc.x, r);
    r = __dp2a_lo((int)bs0.z, (int)sc.y, r);
    r = __dp2a_hi((int)bs0.w, (int)sc.y, r);
    r = __dp2a_lo((int)bs1.x, (int)sc.z, r);
    r = __dp2a_hi((int)bs1.y, (int)sc.z, r);
    r = __dp2a_lo((int)bs1.z, (int)sc.w, r);
    return __dp2a_hi((int)bs1.w, (int)sc.w, r);
}

// One Q6_K super-block (padded 224-byte layout: ql[128] qh[64] int8 sc[16]
// fp16 d at 208) of weight rows a = g, b = g+8 against activation rows g, 2t,
// 2t+1 (Q8_K records: d at 0, quants at 16, int16 16-element sums at 272).
// pix_dot_q6_K (src/kernels_quant.cpp:256-337): value index 128j + 32k + b
// has low bits from ql[64j + 32(k%2) + b] (nibble k/2) and high bits 2k..2k+1
// of qh[32j + b]; scale sc[8j + 2k + b/16].  Each 16-value group is one
// u8 x s8 m16n8k16 MMA on the unsigned 6-bit quants; the -32 offset is the
// reference's separate term 32 * sum_s sc_s * bsum_s.
__device__ __forceinline__ void q6_unit(const uint8_t* wa, const uint8_t* wb, const uint8_t* xg, const uint8_t* x0,
                                        const uint8_t* x1, uint32_t t, float (&acc)[4])
{
    const uint4 sca = *reinterpret_cast<const uint4*>(wa + 192), scb = *reinterpret_cast<const uint4*>(wb + 192);
    int sumi[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 2; j++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t qha = *reinterpret_cast<const uint32_t*>(wa + 128 + 32 * j + 16 * h + 4 * t);
            const uint32_t qhb = *reinterpret_cast<const uint32_t*>(wb + 128 + 32 * j + 16 * h + 4 * t);
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                const uint32_t qla = *reinterpret_cast<const uint32_t*>(wa + 64 * j + 32 * kk + 16 * h + 4 * t);
                const uint32_t qlb = *reinterpret_cast<const uint32_t*>(wb + 64 * j + 32 * kk + 16 * h + 4 * t);
#pragma unroll
                for (int khi = 0; khi < 2; khi++) {
                    const int k = kk + 2 * khi;
                    const uint32_t ha = k == 0 ? qha << 4 : k == 1 ? qha << 2 : k == 2 ? qha : qha >> 2;
                    const uint32_t hb = k == 0 ? qhb << 4 : k == 1 ? qhb << 2 : k == 2 ? qhb : qhb >> 2;
                    const uint32_t aa = ((khi ? qla >> 4 : qla) & 0x0f0f0f0fu) | (ha & 0x30303030u);
                    const uint32_t ab = ((khi ? qlb >> 4 : qlb) & 0x0f0f0f0fu) | (hb & 0x30303030u);
                    const uint32_t bx = *reinterpret_cast<const uint32_t*>(xg + 16 + 128 * j + 32 * k + 16 * h + 4 * t);
                    int d[4];
                    mma_u8s8_k16(d, aa, ab, bx);
                    const int si = 8 * j + 2 * k + h;
                    const int s0 = sbyte(sca, si), s1 = sbyte(scb, si);
                    sumi[0] += s0 * d[0];
                    sumi[1] += s0 * d[1];
                    sumi[2] += s1 * d[2];
                    sumi[3] += s1 * d[3];
                }
            }
        }
    }
    const uint4 b00 = *reinterpret_cast<const uint4*>(x0 + 272), b01 = *reinterpret_cast<const uint4*>(x0 + 288);
    const uint4 b10 = *reinterpret_cast<const uint4*>(x1 + 272), b11 = *reinterpret_cast<const uint4*>(x1 + 288);
    sumi[0] -= 32 * q6_scaled_sums(b00, b01, sca);
    sumi[1] -= 32 * q6_scaled_sums(b10, b11, sca);
    sumi[2] -= 32 * q6_scaled_sums(b00, b01, scb);
    sumi[3] -= 32 * q6_scaled_sums(b10, b11, scb);
    const float dx0 = *reinterpret_cast<const float*>(x0), dx1 = *reinterpret_cast<const float*>(x1);
    const float da = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(wa + 208)));
    const float db = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(wb + 208)));
    // pix_dot_q6_K: d = y.d * fp16(x.d); acc += d * float(sumi - 32 * sum_s sc_s * bsum_s)
    acc[0] = __fmaf_rn(__fmul_rn(dx0, da), (float)sumi[0], acc[0]);
    acc[1] = __fmaf_rn(__fmul_rn(dx1, da), (float)sumi[1], acc[1]);
    acc[2] = __fmaf_rn(__fmul_rn(dx0, db), (float)sumi[2], acc[2]);
    acc[3] = __fmaf_rn(__fmul_rn(dx1, db), (float)sumi[3], acc[3]);
}

// 8 bytes of shared memory at p, where p % 8 == M (M even; the quants of a
// 34-byte Q8_0 block start 2-byte aligned): aligned loads, then funnel shifts.
template <int M>
__device__ __forceinline__ uint2 lds8(const uint8_t* p)
{
    if constexpr (M == 0) {
        return *reinterpret_cast<const uint2*>(p);
    } else if constexpr (M == 4) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(p);
        return make_uint2(w[0], w[1]);
    } else if constexpr (M == 2) {
        const uint2 w01 = *reinterpret_cast<const uint2*>(p - 2);
        const uint32_t w2 = *reinterpret_cast<const uint32_t*>(p + 6);
        return make_uint2(__funnelshift_r(w01.x, w01.y, 16), __funnelshift_r(w01.y, w2, 16));
    } else {
        static_assert(M == 6, "Q8_0 quants are 2-byte aligned");
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(p - 2);
        const uint2 w12 = *reinterpret_cast<const uint2*>(p + 2);
        return make_uint2(__funnelshift_r(w0, w12.x, 16), __funnelshift_r(w12.x, w12.y, 16));
    }
}

// Block J of a 272-byte group (eight raw Q8_0 blocks) of weight rows a = g,
// b = g+8 (16-byte aligned rows): one MMA for the int32 block dots against
// activation rows g (B fragment b0, b1), then pix_dot_q8_0's
// acc += (fp16 dw * fp16 dx) * dot for activation rows 2t, 2t+1.
template <int J>
__device__ __forceinline__ void q8_block(const uint8_t* wa, const uint8_t* wb, uint32_t t, uint32_t b0, uint32_t b1,
                                         float dx0, float dx1, float (&acc)[4])
{
    constexpr int M = (2 * J + 2) & 7;  // alignment of the quants at 34J + 2 (8t keeps it)
    const uint2 qa = lds8<M>(wa + 34 * J + 2 + 8 * t), qb = lds8<M>(wb + 34 * J + 2 + 8 * t);
    const uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
    int d[4];
    mma_s8(d, a, b0, b1);
    const float dwa = __half2float(*reinterpret_cast<const __half*>(wa + 34 * J));
    const float dwb = __half2float(*reinterpret_cast<const __half*>(wb + 34 * J));
    acc[0] = __fmaf_rn(__fmul_rn(dwa, dx0), (float)d[0], acc[0]);
    acc[1] = __fmaf_rn(__fmul_rn(dwa, dx1), (float)d[1], acc[1]);
    acc[2] = __fmaf_rn(__fmul_rn(dwb, dx0), (float)d[2], acc[2]);
    acc[3] = __fmaf_rn(__fmul_rn(dwb, dx1), (float)d[3], acc[3]);
}

// One group of eight Q8_0 blocks (256 values, 272 bytes per row as stored)
// of weight rows a, b against the records of activation rows g (quants, B
// fragments: lane t's eight bytes of blocks 2P, 2P+1 are one 16-byte word)
// and 2t, 2t+1 (block scales, fp32 at byte 256).  The per-element order of
// a block is permuted identically for A and B (lane t: bytes 8t..8t+7).
__device__ __forceinline__ void q8_unit(const uint8_t* wa, const uint8_t* wb, const uint8_t* xg, const uint8_t* x0,
                                        const uint8_t* x1, uint32_t t, float (&acc)[4])
{
    const float4 s0a = *reinterpret_cast<const float4*>(x0 + kQKK), s0b = *reinterpret_cast<const float4*>(x0 + kQKK + 16);
    const float4 s1a = *reinterpret_cast<const float4*>(x1 + kQKK), s1b = *reinterpret_cast<const float4*>(x1 + kQKK + 16);
    const uint8_t* xr = xg + 16 * t;
    uint4 bx = *reinterpret_cast<const uint4*>(xr);
    q8_block<0>(wa, wb, t, bx.x, bx.y, s0a.x, s1a.x, acc);
    q8_block<1>(wa, wb, t, bx.z, bx.w, s0a.y, s1a.y, acc);
    bx = *reinterpret_cast<const uint4*>(xr + 64);
    q8_block<2>(wa, wb, t, bx.x, bx.y, s0a.z, s1a.z, acc);
    q8_block<3>(wa, wb, t, bx.z, bx.w, s0a.w, s1a.w, acc);
    bx = *reinterpret_cast<const uint4*>(xr + 128);
    q8_block<4>(wa, wb, t, bx.x, bx.y, s0b.x, s1b.x, acc);
    q8_block<5>(wa, wb, t, bx.z, bx.w, s0b.y, s1b.y, acc);
    bx = *reinterpret_cast<const uint4*>(xr + 192);
    q8_block<6>(wa, wb, t, bx.x, bx.y, s0b.z, s1b.z, acc);
    q8_block<7>(wa, wb, t, bx.z, bx.w, s0b.w, s1b.w, acc);
}

__device__ __forceinline__ void store_out(const MvParams& p, int64_t r, int64_t col, float v)
{
    p.y[col * p.ldy + r] = p.bias ? __fadd_rn(v, p.bias[r]) : v;
}

// Shared-memory offset of activation row c within a stage: row pitch
// kActPitch plus a skew that grows with c (rows never overlap), chosen so that
// both the B-fragment loads (rows g, g+1 of a quarter warp) and the sum loads
// (rows 2t of four lanes) hit distinct banks: 16 bytes per row pair when the
// pitch is an odd multiple of 64 bytes, else 144 bytes per row pair plus 64
// for odd rows.
template <int TR, uint32_t WT>
__device__ __host__ constexpr uint32_t act_row_off(uint32_t c)
{
    constexpr uint32_t P = kMvStageSuperBlocks / (TR / 16) * MvFmt<WT>::kRecBytes;  // MvShape::kActPitch
    return c * P + (P % 128 == 0 ? 144 * (c >> 1) + 64 * (c & 1) : 16 * (c >> 1));
}
static_assert(act_row_off<16, kTypeQ5_K>(7) + MvShape<16, false, kTypeQ5_K>::kActPitch <= MvShape<16, false, kTypeQ5_K>::kActBytes,
              "activation rows fit the stage");
static_assert(act_row_off<32, kTypeQ5_K>(7) + MvShape<32, false, kTypeQ5_K>::kActPitch <= MvShape<32, false, kTypeQ5_K>::kActBytes,
              "activation rows fit the stage");
static_assert(act_row_off<64, kTypeQ5_K>(7) + MvShape<64, false, kTypeQ5_K>::kActPitch <= MvShape<64, false, kTypeQ5_K>::kActBytes,
              "activation rows fit the stage");
static_assert(act_row_off<16, kTypeQ6_K>(7) + MvShape<16, false, kTypeQ6_K>::kActPitch <= MvShape<16, false, kTypeQ6_K>::kActBytes,
              "activation rows fit the stage");
static_assert(act_row_off<32, kTypeQ6_K>(7) + MvShape<32, false, kTypeQ6_K>::kActPitch <= MvShape<32, false, kTypeQ6_K>::kActBytes,
              "activation rows fit the stage");
static_assert(act_row_off<64, kTypeQ8_0>(7) + MvShape<64, false, kTypeQ8_0>::kActPitch <= MvShape<64, false, kTypeQ8_0>::kActBytes,
              "activation rows fit the stage buffer");
static_assert(act_row_off<32, kTypeQ8_0>(7) + MvShape<32, false, kTypeQ8_0>::kActPitch <= MvShape<32, false, kTypeQ8_0>::kActBytes,
              "activation rows fit the stage buffer");
static_assert(act_row_off<64, kTypeQ6_K>(7) + MvShape<64, false, kTypeQ6_K>::kActPitch <= MvShape<64, false, kTypeQ6_K>::kActBytes,
              "activation rows fit the stage");

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v)
{
    uint32_t old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Sum of the partial sums of tile Tk over its contributing CTAs, in CTA
// order, stored as the tile's outputs; nthr threads (index tid) share the
// tile's outputs, and every contributor's load of an output is in flight
// before the sum.
template <int TR>
__device__ __forceinline__ void mv_tile_sum(const MvParams& p, int64_t Tk, int64_t S, int64_t G, uint32_t spt, uint32_t tid,
                                            uint32_t nthr)
{
    const uint32_t columns = (uint32_t)p.columns;
    const int64_t c_first = cta_of_stage(Tk * spt, S, G), c_last = cta_of_stage((Tk + 1) * spt - 1, S, G);
    const int64_t tile_floats = (int64_t)columns * TR;
    // every contributor after the first starts its range in tile Tk, so its
    // partial sums are in its slot 0; only the first one's slot varies
    const float* first = p.partial + (c_first * 2 + partial_slot(c_first, Tk, S, G, spt)) * tile_floats;
    const float* rest = p.partial + (c_first + 1) * 2 * tile_floats;  // slot 0 of CTA c_first + 1
    const int64_t n_rest = c_last - c_first;
    for (uint32_t idx = tid; idx < columns * TR; idx += nthr) {  // [column][row of the tile]
        float w = __ldcg(first + idx);
        int64_t k = 0;
        for (; k + 8 <= n_rest; k += 8) {
            float pv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) pv[u] = __ldcg(rest + (k + u) * 2 * tile_floats + idx);
#pragma unroll
            for (int u = 0; u < 8; u++) w += pv[u];
        }
        float pv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) pv[u] = k + u < n_rest ? __ldcg(rest + (k + u) * 2 * tile_floats + idx) : 0.f;
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (k + u < n_rest) w += pv[u];
        const int64_t r = Tk * TR + idx % TR;
        if (r < p.rows) store_out(p, r, idx / TR, w);
    }
}

__device__ __forceinline__ int64_t contributors(int64_t Tk, int64_t S, int64_t G, uint32_t spt)
{
    return cta_of_stage((Tk + 1) * spt - 1, S, G) - cta_of_stage(Tk * spt, S, G) + 1;
}

// Fix-up warp: the first tile of this CTA's range, when it is shared with
// other CTAs and is not also the last one.  Waits until the consumers stored
// their partial sums, counts the contribution, and if it is the last one,
// sums all contributions and stores the tile.  Runs while the consumers go on
// with the rest of the range.
template <int TR, bool FUSED, uint32_t WT>
__device__ __forceinline__ void mv_fixup_first(const MvParams& p, MvSmem<TR, FUSED, WT>& sm, int64_t S, int64_t G, uint32_t spt,
                                               uint32_t T0, uint32_t lane)
{
    if (!mbar_wait(&sm.part, 0, &sm.abort, p.status, kDevTimeoutFull)) return;
    // release: the consumers' stores, ordered before by the mbarrier;
    // acquire: the other contributors' stores, for the loads below
    uint32_t last = 0;
    if (lane == 0) last = atom_add_acq_rel_gpu(&p.counters[T0], 1u) == (uint32_t)(contributors(T0, S, G, spt) - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    mv_tile_sum<TR>(p, T0, S, G, spt, lane, 32);
    if (lane == 0) p.counters[T0] = 0u;  // ready for the next call
}

template <int TR, bool FUSED, uint32_t WT>
__global__ void __launch_bounds__(kMvThreads, 2) k_matvec_kq(const __grid_constant__ MvParams p)
{
    using Sh = MvShape<TR, FUSED, WT>;
    constexpr int kStages = Sh::kStages, kSbs = Sh::kSbs, kRg = Sh::kRowGroups;
    constexpr int kRec = MvFmt<WT>::kRecBytes;
    extern __shared__ __align__(128) uint8_t mv_smem[];
    MvSmem<TR, FUSED, WT>& sm = *reinterpret_cast<MvSmem<TR, FUSED, WT>*>(mv_smem);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    griddep_launch_dependents();
    const int64_t G = gridDim.x, c = blockIdx.x, S = p.stages;
    const int64_t s_begin = c * S / G, s_end = (c + 1) * S / G;
    const uint32_t spt = (uint32_t)p.spt, nst = (uint32_t)(s_end - s_begin);
    const uint32_t T0 = (uint32_t)(s_begin / spt), q0 = (uint32_t)(s_begin % spt);  // the only divisions
    const uint32_t nsb = (uint32_t)p.nsb, columns = (uint32_t)p.columns;
    constexpr bool fused = FUSED;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kMvConsumers);
        }
        mbar_init(&sm.part, 32 * kRg);  // every lane of the row-group warps that store partial sums
        sm.abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // Tiles this CTA shares with other CTAs: its first when the range starts
    // inside it or ends before its end, its last when that differs and the
    // range ends before its end.  The fix-up warp finishes a shared first tile
    // that is not also the last; the consumers finish the last one at the end.
    const uint32_t T1 = (uint32_t)((s_end - 1) / spt), q1 = (uint32_t)((s_end - 1) % spt);
    const bool first_shared = q0 != 0 || (T1 == T0 && q1 != spt - 1);
    const bool first_async = first_shared && T1 != T0;
    const bool last_shared = T1 == T0 ? first_shared : q1 != spt - 1;

    if (warp == kMvFixupWarp) {
        if (first_async) {
            griddep_wait();  // counters and partial sums belong to the kernels before this one
            mv_fixup_first<TR, FUSED, WT>(p, sm, S, G, spt, T0, lane);
        }
        return;
    }

    if (warp == kMvProducerWarp) {
        if (lane == 0 && !(p.stall && blockIdx.x == 0)) {
            // producer.  The weights do not depend on earlier kernels: the
            // first stages' weights are requested before griddep_wait, their
            // activation records after it.
            tma_prefetch_desc(&p.map);
            const uint32_t pre = nst < (uint32_t)kStages ? nst : (uint32_t)kStages;
            uint32_t T = T0, q = q0, slot = 0, phase = 0, issued = 0;
            for (uint32_t i = 0; i < nst; i++) {
                if (i >= (uint32_t)kStages && !mbar_wait(&sm.empty[slot], phase ^ 1u, &sm.abort, p.status, kDevTimeoutEmpty))
                    break;
                const uint32_t nsb_here = nsb - kSbs * q < (uint32_t)kSbs ? nsb - kSbs * q : (uint32_t)kSbs;
                const uint32_t act_tx = fused ? 0u : columns * nsb_here * kRec;
                mbar_expect_tx(&sm.full[slot], Sh::kWeightBytes + act_tx);
                // weight tile of logical tile T (gated pairs: gate tile T/2, then up tile T/2)
                const int64_t Tw = p.gated_half ? (int64_t)(T >> 1) + ((T & 1u) ? p.gated_half : 0) : (int64_t)T;
                if (Sh::kRowMajor)
                    tma_load_2d(sm.weight[slot], &p.map, &sm.full[slot], (int32_t)(q * (Sh::kRowBytes / 8)),
                                (int32_t)(p.row_first + Tw * TR));
                else
                    tma_load_3d(sm.weight[slot], &p.map, &sm.full[slot], 0, (int32_t)(p.row_first + Tw * TR),
                                (int32_t)(q * kSbs));
                if (fused) {
                    // the consumers quantize the activation themselves
                } else if (i == pre - 1) {
                    griddep_wait();
                    // activation records of the stages requested so far (slots 0..i)
                    uint32_t qj = q0;
                    for (uint32_t k = 0; k <= i; k++) {
                        const uint32_t nk = nsb - kSbs * qj < (uint32_t)kSbs ? nsb - kSbs * qj : (uint32_t)kSbs;
                        for (uint32_t col = 0; col < columns; col++)
                            bulk_load(sm.act(k) + act_row_off<TR, WT>(col), p.act + ((int64_t)col * nsb + kSbs * qj) * kRec,
                                      nk * kRec, &sm.full[k]);
                        if (++qj == spt) qj = 0;
                    }
                } else if (i >= pre) {
                    for (uint32_t col = 0; col < columns; col++)
                        bulk_load(sm.act(slot) + act_row_off<TR, WT>(col), p.act + ((int64_t)col * nsb + kSbs * q) * kRec,
                                  nsb_here * kRec, &sm.full[slot]);
                }
                issued = i + 1;
                if (++q == spt) { q = 0; T++; }
                if (++slot == (uint32_t)kStages) { slot = 0; phase ^= 1u; }
            }
            // every copy of this CTA lands before it may exit, also after an
            // abort (bounded: a stage that never lands is reported)
            uint32_t never = 0;
            for (uint32_t i = issued > (uint32_t)kStages ? issued - kStages : 0; i < issued; i++)
                mbar_wait(&sm.full[i % kStages], (i / kStages) & 1u, &never, p.status, kDevTimeoutFull);
        }
        return;
    }

    // consumers.
    const uint32_t rg = warp % kRg, sbl = warp / kRg;  // row group, super-block lane
    const uint32_t g = lane >> 2, t = lane & 3u;
    const bool vc0 = 2 * t < columns, vc1 = 2 * t + 1 < columns;  // output columns of this lane
    const uint32_t row_off = (16 * rg + g) * Sh::kRowPitch + sbl * Sh::kSbPitch;
    // Activation, two ways.  Copied per stage: row c of a stage's buffer at
    // act_row_off(c); rows >= columns are never copied, so zero them once and
    // their fragments, sums and scales are zero.  Fused: the records of all
    // of this CTA's stages, [stage][super-block lane][row] x kRec bytes, in
    // the same memory, quantized here from x, plus one zero record for rows
    // >= columns.
    uint8_t* const act_flat = sm.act_area;
    uint8_t* const zero_rec = act_flat + kMvFusedRecords * kRec;
    if (!fused) {
        for (uint32_t k = 0; k < (uint32_t)kStages; k++)
            for (uint32_t c8 = columns; c8 < 8; c8++)
                for (uint32_t o = threadIdx.x * 16; o < (uint32_t)Sh::kActPitch; o += 32 * kMvConsumers * 16)
                    *reinterpret_cast<uint4*>(sm.act(k) + act_row_off<TR, WT>(c8) + o) = make_uint4(0, 0, 0, 0);
    } else if (threadIdx.x < kRec / 16) {
        reinterpret_cast<uint4*>(zero_rec)[threadIdx.x] = make_uint4(0, 0, 0, 0);
    }
    // outputs, partials, counters and x belong to the kernels before this one
    griddep_wait();
    if (fused) {
        // this warp's tasks (at most kMvFusedRecords / 8): every load in
        // flight before the first block is quantized
        constexpr int kPerWarp = kMvFusedRecords / kMvConsumers;
        const uint32_t per_stage = kSbs * columns, ntask = nst * per_stage;
        float v[kPerWarp][8];
        uint32_t sbk[kPerWarp];
#pragma unroll
        for (int k = 0; k < kPerWarp; k++) {
            const uint32_t task = warp + kMvConsumers * k;
            const uint32_t i = task / per_stage, rem = task % per_stage;
            const uint32_t lane_sb = rem / columns, c = rem % columns;
            sbk[k] = task < ntask ? kSbs * ((q0 + i) % spt) + lane_sb : nsb;  // >= nsb: nothing to do
            if (sbk[k] < nsb) q8_K_load(p.x + (int64_t)c * p.ldx + (int64_t)sbk[k] * kQKK, lane, v[k]);
        }
#pragma unroll
        for (int k = 0; k < kPerWarp; k++) {
            if (sbk[k] >= nsb) continue;  // warp-uniform; past the end of K the record is never read
            if constexpr (WT == kTypeQ8_0) {
                q8_0_store_mv(act_flat + (warp + kMvConsumers * k) * kRec, v[k], lane);
            } else {
                const Q8KWarp r = q8_K_warp_vals(v[k], lane);
                if constexpr (WT == kTypeQ5_K)
                    q8_K_store_mv(act_flat + (warp + kMvConsumers * k) * kRec, r, lane);
                else
                    q8_K_store_q6(act_flat + (warp + kMvConsumers * k) * kRec, r, lane);
            }
        }
    }
    named_bar_sync(7, 32 * kMvConsumers);
    const uint32_t xg_off = act_row_off<TR, WT>(g) + sbl * kRec;          // record of activation row g
    const uint32_t x0_off = act_row_off<TR, WT>(2 * t) + sbl * kRec;      // activation row 2t
    const uint32_t x1_off = act_row_off<TR, WT>(2 * t + 1) + sbl * kRec;  // activation row 2t+1
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, summ[4] = {0.f, 0.f, 0.f, 0.f};
    float gate_v[4] = {0.f, 0.f, 0.f, 0.f};  // gated pairs: the gate tile's sums, until the up tile ends
    bool ok = true;
    uint32_t seg = 0, slot = 0, phase = 0, T = T0, q = q0;
    bool seg_whole_start = q0 == 0;  // this segment starts at its tile's first stage
    for (uint32_t i = 0; i < nst; i++) {
        const uint32_t sb = kSbs * q + sbl;
        if (ok) ok = mbar_wait(&sm.full[slot], phase, &sm.abort, p.status, kDevTimeoutFull);
        if (ok && sb < nsb) {
            const uint8_t* wa = sm.weight[slot] + row_off;
            const uint8_t* wb = wa + 8 * Sh::kRowPitch;
            const uint8_t *xg, *x0, *x1;  // records of activation rows g, 2t, 2t+1
            if (!fused) {
                xg = sm.act(slot) + xg_off;
                x0 = sm.act(slot) + x0_off;
                x1 = sm.act(slot) + x1_off;
            } else {
                const uint8_t* rec = act_flat + (i * kSbs + sbl) * columns * kRec;
                xg = g < columns ? rec + g * kRec : zero_rec;
                x0 = vc0 ? rec + 2 * t * kRec : zero_rec;
                x1 = vc1 ? rec + (2 * t + 1) * kRec : zero_rec;
            }
            if constexpr (WT == kTypeQ5_K)
                q5_unit(wa, wb, xg, x0, x1, t, acc, summ);
            else if constexpr (WT == kTypeQ6_K)
                q6_unit(wa, wb, xg, x0, x1, t, acc);
            else
                q8_unit(wa, wb, xg, x0, x1, t, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[slot]);
        if (++slot == (uint32_t)kStages) { slot = 0; phase ^= 1u; }
        const bool tile_last = q == spt - 1;
        const uint32_t Tcur = T;
        if (++q == spt) { q = 0; T++; }
        if (!tile_last && i != nst - 1) continue;

        // ---- end of this CTA's segment of tile Tcur ----
        float v[4] = {acc[0] + summ[0], acc[1] + summ[1], acc[2] + summ[2], acc[3] + summ[3]};
        // lanes >= 1 hand their sums to lane 0 through a buffer alternating
        // by segment: before one can write it again, lane 0 has passed the
        // next segment's barrier, i.e. finished reading it
        float (*red)[kRg][16][8] = sm.red[seg & 1u];
        if (sbl > 0) {
            red[sbl - 1][rg][g][2 * t] = v[0];
            red[sbl - 1][rg][g][2 * t + 1] = v[1];
            red[sbl - 1][rg][g + 8][2 * t] = v[2];
            red[sbl - 1][rg][g + 8][2 * t + 1] = v[3];
        }
        named_bar_sync(1 + rg, 32 * kSbs);
        if (sbl == 0) {
#pragma unroll
            for (int k = 0; k < kSbs - 1; k++) {  // fixed order: lane 0, 1, 2, ...
                v[0] += red[k][rg][g][2 * t];
                v[1] += red[k][rg][g][2 * t + 1];
                v[2] += red[k][rg][g + 8][2 * t];
                v[3] += red[k][rg][g + 8][2 * t + 1];
            }
            const int64_t ra = (int64_t)Tcur * TR + 16 * rg + g, rb = ra + 8;
            if (p.gated_half) {
                // whole tiles in pairs: keep the gate sums, then finish tensor_silu +
                // tensor_gate on the up sums of the same rows (the order of operations
                // of the two-kernel path)
                if ((Tcur & 1u) == 0) {
#pragma unroll
                    for (int k = 0; k < 4; k++) gate_v[k] = v[k];
                } else {
                    const int64_t na = (int64_t)(Tcur >> 1) * TR + 16 * rg + g, nb = na + 8;
                    float o[4];
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        o[k] = __fmul_rn(__fdiv_rn(gate_v[k], __fadd_rn(1.0f, expf(-gate_v[k]))), v[k]);
                    if (vc0) p.y[(int64_t)(2 * t) * p.ldy + na] = o[0];
                    if (vc1) p.y[(int64_t)(2 * t + 1) * p.ldy + na] = o[1];
                    if (vc0) p.y[(int64_t)(2 * t) * p.ldy + nb] = o[2];
                    if (vc1) p.y[(int64_t)(2 * t + 1) * p.ldy + nb] = o[3];
                }
            } else if (seg_whole_start && tile_last) {
                if (vc0 && ra < p.rows) store_out(p, ra, 2 * t, v[0]);
                if (vc1 && ra < p.rows) store_out(p, ra, 2 * t + 1, v[1]);
                if (vc0 && rb < p.rows) store_out(p, rb, 2 * t, v[2]);
                if (vc1 && rb < p.rows) store_out(p, rb, 2 * t + 1, v[3]);
            } else {
                // partial sums of this segment for the fix-up warp
                float* mine = p.partial + (c * 2 + partial_slot(c, Tcur, S, G, spt)) * columns * TR;
                const uint32_t la = 16 * rg + g, lb = la + 8;
                if (vc0) {
                    mine[(2 * t) * TR + la] = v[0];
                    mine[(2 * t) * TR + lb] = v[2];
                }
                if (vc1) {
                    mine[(2 * t + 1) * TR + la] = v[1];
                    mine[(2 * t + 1) * TR + lb] = v[3];
                }
                if (seg == 0 && first_async) mbar_arrive(&sm.part);  // each lane releases its own stores
            }
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        summ[0] = summ[1] = summ[2] = summ[3] = 0.f;
        seg++;
        seg_whole_start = true;  // later segments start at a tile's first stage
    }

    // ---- the range's last tile, when shared: count, and the last contributor
    // sums it with all consumer threads.  The row-group lane-0 warps' stores
    // are ordered before the count by the barrier and thread 0's release, the
    // loads after its acquire by the second barrier. ----
    if (!last_shared) return;
    named_bar_sync(6, 32 * kMvConsumers);
    if (threadIdx.x == 0)
        sm.last = atom_add_acq_rel_gpu(&p.counters[T1], 1u) == (uint32_t)(contributors(T1, S, G, spt) - 1);
    named_bar_sync(6, 32 * kMvConsumers);
    if (!sm.last) return;
    mv_tile_sum<TR>(p, T1, S, G, spt, threadIdx.x, 32 * kMvConsumers);
    if (threadIdx.x == 0) p.counters[T1] = 0u;  // ready for the next call
}

template <int TR, bool FUSED, uint32_t WT>
cudaError_t launch_kq(const MatvecPlan& plan, const CUtensorMap* map, int64_t row_first, const void* act, const float* x,
                      int64_t ldx, float* y, int64_t ldy, const float* bias, float* partial, uint32_t* counters,
                      uint32_t* status, cudaStream_t s)
{
    static std::atomic<bool> attr_set[16] = {};  // set once per device (racing threads set the same values)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && !attr_set[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(k_matvec_kq<TR, FUSED, WT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(MvSmem<TR, FUSED, WT>));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_matvec_kq<TR, FUSED, WT>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        attr_set[dev].store(true, std::memory_order_release);
    }
    MvParams prm;
    prm.map = *map;
    prm.act = static_cast<const uint8_t*>(act);
    prm.x = x;
    prm.ldx = ldx;
    prm.y = y;
    prm.bias = bias;
    prm.partial = partial;
    prm.counters = counters;
    prm.status = status;
    prm.ldy = ldy;
    prm.rows = plan.rows;
    prm.row_first = row_first;
    prm.stages = plan.stages;
    prm.nsb = (int32_t)(plan.inner / kQKK);
    prm.spt = (int32_t)plan.spt;
    prm.columns = (int32_t)plan.columns;
    prm.gated_half = plan.gated_half;
    prm.stall = plan.debug_stall ? 1 : 0;
    return launch_pdl(k_matvec_kq<TR, FUSED, WT>, dim3(plan.grid), dim3(kMvThreads), sizeof(MvSmem<TR, FUSED, WT>), s, prm);
}

// The kernel instance for a plan: weight format x fused quantize.
template <int TR>
cudaError_t launch_kq3(const MatvecPlan& plan, const CUtensorMap* map, int64_t row_first, const void* act, const float* x,
                       int64_t ldx, float* y, int64_t ldy, const float* bias, float* partial, uint32_t* counters,
                       uint32_t* status, cudaStream_t s)
{
    if (plan.type == kTypeQ8_0) {
        // 16-row tiles only with the fused quantize: two CTAs of the unfused
        // variant (per-stage activation buffers) do not fit one SM
        if constexpr (TR == 16) {
            if (!plan.fused) return cudaErrorInvalidValue;
            return launch_kq<16, true, kTypeQ8_0>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
        } else {
            return plan.fused ? launch_kq<TR, true, kTypeQ8_0>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s)
                              : launch_kq<TR, false, kTypeQ8_0>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
        }
    }
    if (plan.type == kTypeQ5_K)
        return plan.fused ? launch_kq<TR, true, kTypeQ5_K>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s)
                          : launch_kq<TR, false, kTypeQ5_K>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
    return plan.fused ? launch_kq<TR, true, kTypeQ6_K>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s)
                      : launch_kq<TR, false, kTypeQ6_K>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
}

}  // namespace

int matvec_map_index(int tile_rows) { return tile_rows == 64 ? 0 : tile_rows == 32 ? 1 : 2; }

MatvecPlan plan_matvec(uint32_t type, int64_t rows, int64_t inner, int64_t columns, int num_sms, bool fuse_quantize,
                       bool gated)
{
    MatvecPlan p;
    p.type = type;
    p.rows = rows;
    p.inner = inner;
    p.columns = columns;
    const bool q8 = type == kTypeQ8_0;
    if (type == kTypeQ5_K || type == kTypeQ6_K || (q8 && inner % kQKK == 0)) {
        // the TMA-fed kernel; Q8_0 rows stream as groups of eight blocks
        // (272 bytes), which needs whole groups (and so 16-byte row strides)
        p.streamed = true;
        const int64_t nsb = inner / kQKK;
        const int64_t sb_bytes = type == kTypeQ5_K ? kQ5KBytes : q8 ? kQ80SbBytes : kQ6KPadBytes;
        const int64_t rec_bytes = type == kTypeQ5_K ? kQ8KMvBytes : q8 ? kQ80MvBytes : kQ8KQ6Bytes;
        const int64_t slots = (int64_t)num_sms * 2;  // two CTAs per SM
        // Whole tiles per CTA (no cross-CTA sums) when some tile height gives
        // a tile count that fills the grid well, or when the matrix is small
        // enough that the extra wave costs less than the cross-CTA sums (for
        // Q5_K, 16-row tiles at any length: measured faster than stream-K on
        // the 3584 x 18944 down projection); otherwise 64-row tiles in a
        // stream-K split over the whole grid.
        p.tile_rows = 64;
        bool whole = false;
        // gated: 64-row tiles taken in pairs (gate tile j, up tile j) by one CTA each
        if (gated) p.gated_half = rows / 128;
        for (int tr : {64, 32, 16}) {
            if (gated) break;
            // Q8_0: 16-row tiles only when every CTA quantizes its own records
            if (q8 && tr == 16 && !(fuse_quantize && columns * ((nsb + 7) / 8) * 8 <= kMvFusedRecords)) continue;
            const int64_t tiles = (rows + tr - 1) / tr;
            const int64_t tile_bytes = (int64_t)tr * nsb * sb_bytes;
            const bool short_tiles = tile_bytes <= 64 * 1024 || (type == kTypeQ5_K && tr == 16);
            if (tiles <= slots && (tiles * 20 >= slots * 19 || (tiles * 4 >= slots * 3 && short_tiles))) {
                p.tile_rows = tr;
                whole = true;
                break;
            }
        }
        const int sbs = kMvStageSuperBlocks / (p.tile_rows / 16);
        p.tiles = (rows + p.tile_rows - 1) / p.tile_rows;
        p.spt = (nsb + sbs - 1) / sbs;
        p.stages = p.tiles * p.spt;
        p.grid = (int)(gated ? p.tiles / 2 : whole ? p.tiles : (p.stages < slots ? p.stages : slots));
        // small activations: every CTA quantizes the records of its own stages
        // (at most kMvFusedRecords), no separate quantize kernel
        const int64_t max_stages = (p.stages + p.grid - 1) / p.grid;
        p.fused = fuse_quantize && columns * max_stages * sbs <= kMvFusedRecords;
        p.act_bytes = p.fused ? 0 : (size_t)(columns * nsb * rec_bytes);
        p.partial_bytes = whole || gated ? 0 : (size_t)p.grid * 2 * columns * p.tile_rows * sizeof(float);
        p.counter_bytes = (size_t)p.tiles * sizeof(uint32_t);
    } else {
        const int64_t nblocks = inner / kQK8_0;
        const int64_t min_chunk = 32;  // keep every warp busy on a slice
        p.rowgroups = (rows + kRowsPerCta - 1) / kRowsPerCta;
        // enough CTAs to cover every SM a few times
        const int64_t target = (int64_t)num_sms * 4;
        int64_t ks = (target + p.rowgroups - 1) / p.rowgroups;
        const int64_t max_ks_work = nblocks / min_chunk > 1 ? nblocks / min_chunk : 1;
        if (ks > max_ks_work) ks = max_ks_work;
        if (ks < 1) ks = 1;
        const int64_t chunk = (nblocks + ks - 1) / ks;
        ks = (nblocks + chunk - 1) / chunk;
        p.ks = (int)ks;
        p.chunk = (int)chunk;
        p.grid = (int)(p.rowgroups * ks);
        // + 64: the 2-byte-aligned activation reads may touch a few bytes past the last block
        p.act_bytes = (size_t)(columns * nblocks * kQ8_0Bytes) + 64;
        p.partial_bytes = ks > 1 ? (size_t)ks * columns * rows * sizeof(float) : 0;
        p.counter_bytes = ks > 1 ? (size_t)p.rowgroups * sizeof(uint32_t) : 0;
    }
    // The counters sit at the start of the scratch, in a region that only ever
    // holds counters; calls leave them zero, so a fused call (no quantize
    // kernel to clear them) finds zeros there whatever the previous call was.
    if (p.fused && p.counter_bytes > kMvCounterRegion) {
        p.fused = false;
        p.act_bytes = (size_t)(columns * (inner / kQKK) *
                               (type == kTypeQ5_K ? kQ8KMvBytes : type == kTypeQ8_0 ? kQ80MvBytes : kQ8KQ6Bytes));
    }
    p.off_counters = 0;
    p.off_act = (p.counter_bytes > kMvCounterRegion ? p.counter_bytes + 255 : kMvCounterRegion) / 256 * 256;
    p.off_partial = (p.off_act + p.act_bytes + 255) / 256 * 256;
    p.total_bytes = p.off_partial + p.partial_bytes;
    return p;
}

cudaError_t launch_matvec(const MatvecPlan& plan, const CUtensorMap* maps, int64_t row_first, const uint8_t* w,
                          int64_t stride, const void* act, const float* x, int64_t ldx, float* y, int64_t ldy,
                          const float* bias, float* partial, uint32_t* counters, uint32_t* status, cudaStream_t s)
{
    if (plan.columns < 1 || plan.columns > 8 || plan.grid < 1) return cudaErrorInvalidValue;
    if (plan.streamed) {
        if (!maps || !counters || (plan.partial_bytes && !partial)) return cudaErrorInvalidValue;
        if (plan.fused ? !x : !act) return cudaErrorInvalidValue;
        const CUtensorMap* map = maps + matvec_map_index(plan.tile_rows);
        switch (plan.tile_rows) {
        case 64: return launch_kq3<64>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
        case 32: return launch_kq3<32>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
        case 16: return launch_kq3<16>(plan, map, row_first, act, x, ldx, y, ldy, bias, partial, counters, status, s);
        default: return cudaErrorInvalidValue;
        }
    }
    if (plan.type == kTypeQ8_0) {
        if (plan.fused || (plan.ks > 1 && (!partial || !counters))) return cudaErrorInvalidValue;
        return launch_pdl(k_matvec_q8_0, dim3(plan.grid), dim3(kThreads), 0, s, w, stride, plan.rows, plan.inner,
                          static_cast<const uint8_t*>(act), plan.columns, y, ldy, bias, plan.ks, plan.chunk, partial,
                          counters);
    }
    return cudaErrorInvalidValue;
}

}  // namespace pxq
