// gemm.cu -- large-M K-quant (Q5_K, Q6_K) GEMM on the 5th-generation
// tensor cores, one CTA pair per output tile.  (Q8_0: gemm_q8.cu.)
//
// Computes Y[m, n] = sum over K-blocks b of  s(m,n,b) * I(m,n,b)
// where I is the exact integer dot of one block of quants and s the product
// of the block scales -- the arithmetic of pix_dot_q5_K
// (src/kernels_quant.cpp:163-254) and pix_dot_q6_K (:256-337) as driven by
// cpu_quant_matmul (:389-400), for every (activation row m, weight row n).
//
// Design (sm_100a):
//   * Operands are exact fp16 copies of the int8 quants (activations from
//     quantize.cu, weights from the one-time repack in repack.cu) with the
//     sub-block scales folded into the weight side.  A kind::f16 tcgen05.mma
//     with fp32 accumulation computes each 64-value chunk dot exactly
//     (< 2^24) and hands the drain a float; the folded scales make the
//     chunk values larger than int8, so kind::i8 does not apply.
//   * CTA pairs (cta_group::2): the two CTAs of a cluster share every MMA.
//     The pair's tile is 256 weight rows (the MMA's M; each CTA stages and
//     accumulates its 128) by TMP activation rows (the MMA's N; each CTA
//     stages TMP/2 of them and receives all TMP columns in its TMEM).  Per
//     FLOP each CTA moves half the operand bytes of a one-CTA 128-row tile,
//     which is what bounds that design: the operand stream into shared
//     memory and the MMA's reads of it share one memory.
//     The even CTA issues the MMAs; both CTAs' TMA loads report on its stage
//     barriers; its commits arrive on the barriers of both CTAs; the odd
//     CTA's drain warps release accumulator slots on the even CTA's
//     barriers.
//   * Orientation: TMEM lanes are WEIGHT rows, TMEM columns are ACTIVATION
//     rows.  Per-weight-row scales are then per-thread scalars, and the 32
//     lanes of a warp store 32 consecutive outputs.
//   * Q5_K (TMP = 256, two 256-column slots): 6-bit sub-block scales are
//     folded into the weight operand (sc*q5 <= 1953, exact in fp16), so every
//     64-value chunk dot is exact in the fp32 accumulator, and the four
//     chunks of a super-block, which share its scale dW*dX, accumulate into
//     one slot.  Their sum is exact while it stays below 2^24 in magnitude
//     (always, for real activations; the reference rounds its int32 sum to
//     fp32 once).  The min term sum_j m_j*bsum_j is a K=16 MMA per
//     super-block on exact (hi, lo) splits into the other slot; the two slots
//     swap roles every super-block, and the min MMA is issued after the
//     third chunk stage, so the drain of the previous super-block's chunk
//     sum overlaps three stages of MMAs.
//   * Q6_K (TMP = 256, two slots alternating per super-block): the 8-bit
//     scale and the -32 offset fold into v = sc*(q6-32), |v| <= 4096 -- odd
//     values above 2048 need one bit more than fp16 has, so the repack keeps
//     an even plane (exact in fp16) and a parity plane, two MMAs per K step
//     into the same slot.  No min term; one drain per super-block.
//   * The block-dot dump (pxq_gemm_block_dots) drains every block / chunk /
//     min sum on its own, so the exact int32 dots stay checkable.
//   * Warp roles (12 warps, 3 warpgroups): warpgroups 0-1 drain TMEM (warp w
//     reads lane quadrant w%4 and column half w/4) with 224 registers
//     (setmaxnreg); warpgroup 2 runs the TMA producer (warp 8, every CTA)
//     and the single-thread MMA issuer (warp 9 of the even CTA) with 40-56,
//     within the 384*168 registers the block launches with.
//     Persistent pairs walk the output tiles.
//   * Every mbarrier wait is bounded (pxq_device.cuh).  Every CTA loads its
//     own tiles from this GPU's HBM into its own shared memory; no cluster
//     broadcast of any load.
#include <cuda.h>
#include <mutex>
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int TN = 128;                // weight rows per CTA (TMEM lanes); the pair's MMA M is 256
constexpr int BK = 64;                 // fp16 K elements per stage (128-byte rows)
constexpr int W_BYTES = TN * BK * 2;   // 16 KB
constexpr int SW32_W = TN * 32;        // [128][16] fp16 tile, 32-byte swizzle: 4 KB
constexpr int DRAIN_WARPS = 8;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int THREADS = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr int MAX_STAGES = 6;
constexpr int DEPTH = 2;               // min-operand ring
constexpr int MAX_SB_DEPTH = 4;        // super-block scale entry ring (per type: Cfg::SB_DEPTH)

template <uint32_t TYPE>
struct Cfg;
template <>
struct Cfg<kTypeQ5_K> {
    static constexpr int CG = 2, TMP = 256, SLOTS = 2, STAGES = 4;
    static constexpr uint32_t PRODUCER_REGS = 56, DRAIN_REGS = 224;
    static constexpr int SROWS = 64;  // activation rows per TMA store of a drain warp
    static constexpr int XR = TMP / CG, X_BYTES = XR * BK * 2, SW32_X = XR * 32;
    static constexpr int STAGE = W_BYTES + X_BYTES;                          // 32 KB
    static constexpr int MIN_ENTRY = SW32_W + SW32_X;                        // weight | activation min operands
    static constexpr int SB_ENTRY = 2048, SB_DEPTH = 2;                      // dW | dminW | dX (TMP floats)
    static constexpr int OFF_DW = 0, OFF_DMW = 512, OFF_DX = 1024;
};
template <>
struct Cfg<kTypeQ6_K> {
    static constexpr int CG = 2, TMP = 256, SLOTS = 2, STAGES = 3;
    static constexpr uint32_t PRODUCER_REGS = 56, DRAIN_REGS = 224;
    static constexpr int SROWS = 64;
    static constexpr int XR = TMP / CG, X_BYTES = XR * BK * 2;
    static constexpr int STAGE = 2 * W_BYTES + X_BYTES;                      // even | parity | X: 48 KB
    static constexpr int MIN_ENTRY = 0;
    // an entry is freed only when the drain has finished its super-block, one
    // super-block after its MMAs: four entries keep the producer clear of the drain
    static constexpr int SB_ENTRY = 2048, SB_DEPTH = 4;                      // dW | dX (TMP floats)
    static constexpr int OFF_DW = 0, OFF_DMW = 0, OFF_DX = 1024;
};

template <uint32_t TYPE>
__host__ __device__ constexpr int off_min() { return Cfg<TYPE>::STAGES * Cfg<TYPE>::STAGE; }
template <uint32_t TYPE>
__host__ __device__ constexpr int off_sb() { return off_min<TYPE>() + DEPTH * Cfg<TYPE>::MIN_ENTRY; }
template <uint32_t TYPE>
__host__ __device__ constexpr int off_staging() { return off_sb<TYPE>() + Cfg<TYPE>::SB_DEPTH * Cfg<TYPE>::SB_ENTRY; }
// output staging for the TMA-store epilogue: per drain warp [SROWS activation rows][32 weight rows] fp32
template <uint32_t TYPE>
__host__ __device__ constexpr int staging_bytes() { return DRAIN_WARPS * Cfg<TYPE>::SROWS * 32 * 4; }
template <uint32_t TYPE>
__host__ __device__ constexpr int off_bar() { return off_staging<TYPE>() + staging_bytes<TYPE>(); }
// full/empty, min full/empty, entry full/empty, slot full/empty, MMA drain-out, gated hand-over
constexpr int NUM_BARS = 2 * MAX_STAGES + 2 * DEPTH + 2 * MAX_SB_DEPTH + 2 * 4 + 1 + 2;
template <uint32_t TYPE>
__host__ __device__ constexpr int smem_bytes() { return off_bar<TYPE>() + NUM_BARS * 8 + 16 + 1024; }

// register split: two drain warpgroups and the producer warpgroup within the
// 384 x 168 registers the block launches with
template <uint32_t TYPE>
constexpr bool regs_fit() { return 256 * Cfg<TYPE>::DRAIN_REGS + 128 * Cfg<TYPE>::PRODUCER_REGS <= 384 * 168; }
static_assert(regs_fit<kTypeQ5_K>() && regs_fit<kTypeQ6_K>(), "setmaxnreg split");
static_assert(Cfg<kTypeQ5_K>::STAGES <= MAX_STAGES && Cfg<kTypeQ6_K>::STAGES <= MAX_STAGES, "stage count");
static_assert(smem_bytes<kTypeQ5_K>() <= 232448, "Q5_K shared memory");
static_assert(smem_bytes<kTypeQ6_K>() <= 232448, "Q6_K shared memory");
static_assert(Cfg<kTypeQ5_K>::STAGE % 1024 == 0 && Cfg<kTypeQ6_K>::STAGE % 1024 == 0 &&
                  Cfg<kTypeQ5_K>::MIN_ENTRY % 1024 == 0 && Cfg<kTypeQ5_K>::SB_ENTRY % 1024 == 0,
              "swizzled tiles need 1024-byte alignment");
static_assert(Cfg<kTypeQ5_K>::SLOTS * Cfg<kTypeQ5_K>::TMP <= (int)TMEM_COLS && Cfg<kTypeQ6_K>::SLOTS * Cfg<kTypeQ6_K>::TMP <= (int)TMEM_COLS,
              "TMEM columns");

struct Params {
    int64_t M, N, K;
    int64_t n_first;
    float* y;
    int64_t ldy;
    const float* bias;
    float* dump;
    uint32_t* status;
    int tma_store;  // 1: epilogue through shared memory + TMA store (tmY)
    int gated;      // 1: gated weight, y = silu(gate) * up over N/2 outputs (direct stores)
    int ndst;       // scatter: also store element (m, n) at ydst[k][m * ldy + col_off + n], k < ndst
    int dst_vec4;   // scatter: every ydst[k] + col_off 16-byte aligned and ldy % 4 == 0 (4-float stores)
    int64_t col_off;
    float* ydst[kMaxScatter];
};

// One output element: this GPU's y and, for a scatter, the same element in
// every peer's buffer (plain stores over NVLink).
__device__ __forceinline__ void put_y(const Params& p, int64_t m, int64_t n, float v)
{
    p.y[m * p.ldy + n] = v;
    const int64_t off = m * p.ldy + p.col_off + n;
    for (int k = 0; k < p.ndst; k++) p.ydst[k][off] = v;
}

// tcgen05 and stage-load forms for a CTA pair (CG = 2); a kernel uses one
// form throughout, as tcgen05 requires.
template <int CG>
struct Grp;
template <>
struct Grp<2> {
    static __device__ __forceinline__ void alloc(uint32_t* dst, uint32_t n) { tmem_alloc_pair(dst, n); }
    static __device__ __forceinline__ void relinquish() { tmem_relinquish_pair(); }
    static __device__ __forceinline__ void dealloc(uint32_t t, uint32_t n) { tmem_dealloc_pair(t, n); }
    static __device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
    {
        mma_f16_pair(d, a, b, idesc, acc);
    }
    static __device__ __forceinline__ void commit(uint64_t* bar) { mma_commit_pair(bar); }
    static __device__ __forceinline__ void commit_local(uint64_t* bar) { mma_commit_pair_local(bar); }
    // stage load reporting on the even CTA's barrier (cluster address)
    static __device__ __forceinline__ void load(void* dst, const void* map, uint64_t*, uint32_t bar, int32_t c0, int32_t c1)
    {
        tma_load_2d_pair(dst, map, bar, c0, c1);
    }
    static __device__ __forceinline__ void sync() { cluster_sync(); }
};

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }
__device__ __forceinline__ uint64_t desc_sw32(uint32_t saddr) { return smem_desc(saddr, 16, 256, 6); }

// K-quant accumulators use the 16x256b TMEM layout: a drain warp covers its
// 32 lanes x 128 columns as acc[((ch*2 + lh)*8 + k)*4 + 2h + c] = lane
// 16lh + 8h + t/4, column 64ch + 8k + 2(t%4) + c (t = lane id).  Each thread
// then needs 32 per-column activation scales (not 128) and 4 per-lane weight
// scales.
__host__ __device__ constexpr int split_idx(int ch, int lh, int k, int h, int c) { return (((ch * 2 + lh) * 8 + k) * 4) + 2 * h + c; }

// acc += (dx[column] * w[lane]) * v over one drained item (taddr: the warp's
// lane quadrant and first column; dx: the warp's first column's scale;
// w4 components x, y, z, w: the scales of lanes t/4, 8 + t/4, 16 + t/4, 24 + t/4).
__device__ __forceinline__ void drain_split(float (&acc)[128], uint32_t taddr, const float* dx, float4 w4, uint32_t t)
{
#pragma unroll
    for (int ch = 0; ch < 2; ch++) {
#pragma unroll
        for (int lh = 0; lh < 2; lh++) {
            uint32_t v[32];
            tmem_ld16x256_x8(taddr + ((16u * lh) << 16) + 64u * ch, v);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 8; k++) {
                // re-read per lane half: keeps the drain's live registers below its budget
                const float2 d = *reinterpret_cast<const float2*>(dx + 64 * ch + 8 * k + 2 * (t & 3));
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const float w = (2 * lh + h) == 0 ? w4.x : (2 * lh + h) == 1 ? w4.y : (2 * lh + h) == 2 ? w4.z : w4.w;
                    float s0, s1;
                    fmul2(s0, s1, d.x, d.y, w, w);
                    const int i = split_idx(ch, lh, k, h, 0);
                    ffma2(acc[i], acc[i + 1], s0, s1, __uint_as_float(v[4 * k + 2 * h]), __uint_as_float(v[4 * k + 2 * h + 1]));
                }
            }
        }
    }
}

// Store one drained item as raw block dots (pxq_gemm_block_dots).
template <int HC>
__device__ __forceinline__ void drain_dump(uint32_t taddr, const Params& p, int64_t item, int64_t m_first, int64_t n)
{
#pragma unroll 1
    for (int g = 0; g < HC / 32; g++) {
        uint32_t v[32];
        tmem_ld32(taddr + 32u * g, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int64_t m = m_first + 32 * g + j;
            if (n < p.N && m < p.M) p.dump[(item * p.M + m) * p.N + n] = __uint_as_float(v[j]);
        }
    }
}

// tensor maps:
//   tmW   weight operand fp16 [N][K] (Q6_K: [N][2K])  box {64, 128}  128B swizzle
//   tmX   activation operand fp16 [M][K]               box {64, TMP/2} 128B swizzle
//         tmXs  activation scales fp16 [M][nb]          box {16, TMP/2} 32B swizzle
//   Q5_K: tmWs  weight min operand fp16 [N][nsb*16]     box {16, 128} 32B swizzle
//         tmXs  activation min operand fp16 [M][nsb*16] box {16, TMP/2} 32B swizzle
//         tmD   weight d   fp32 [nsb][N4]  box {128, 1}
//         tmDm  weight dmin fp32 [nsb][N4] box {128, 1}
//         tmDx  activation d fp32 [nsb][M4] box {TMP, 1}
//   Q6_K: tmD, tmDx as for Q5_K (the others unused)
template <uint32_t TYPE, bool DUMP>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
           const __grid_constant__ CUtensorMap tmWs, const __grid_constant__ CUtensorMap tmXs,
           const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmDm,
           const __grid_constant__ CUtensorMap tmDx, const __grid_constant__ CUtensorMap tmY, const Params p)
{
    using C = Cfg<TYPE>;
    using G = Grp<C::CG>;
    constexpr int CG = C::CG;
    constexpr bool Q5 = TYPE == kTypeQ5_K;
    constexpr bool Q6 = TYPE == kTypeQ6_K;
    constexpr int TMP = C::TMP, XR = C::XR, STAGES = C::STAGES;
    constexpr int HC = TMP / 2;  // TMEM columns per drain warp
    static_assert(HC == 128, "the 16x256b accumulator layout covers 128 columns per warp");
    constexpr uint32_t IDESC = idesc_f16_f32(CG * TN, TMP);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + off_bar<TYPE>());
    uint64_t* full = bars;                   // even CTA: stage loaded (both CTAs' bytes)
    uint64_t* empty = bars + MAX_STAGES;     // stage consumed (both CTAs)
    uint64_t* mfull = empty + MAX_STAGES;    // even CTA: min operands loaded (both CTAs' bytes)
    uint64_t* mempty = mfull + DEPTH;        // min operands consumed (both CTAs)
    uint64_t* sfull = mempty + DEPTH;        // this CTA's super-block scale entry loaded
    uint64_t* sempty = sfull + MAX_SB_DEPTH; // ... and read by this CTA's drain warps
    uint64_t* tfull = sempty + MAX_SB_DEPTH; // accumulator slot complete (both CTAs)
    uint64_t* tempty = tfull + 4;            // even CTA: slot drained by both CTAs
    uint64_t* mma_done = tempty + 4;         // even CTA: every issued MMA finished (exit path)
    uint64_t* merge = mma_done + 1;          // gated epilogue: hand-over buffer free / written
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    uint8_t* min_region = smem + off_min<TYPE>();
    uint8_t* sb_region = smem + off_sb<TYPE>();

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < MAX_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < DEPTH; i++) {
            mbar_init(&mfull[i], 1);
            mbar_init(&mempty[i], 1);
        }
        for (int i = 0; i < MAX_SB_DEPTH; i++) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sempty[i], DRAIN_WARPS);
        }
        for (int i = 0; i < 4; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], CG * DRAIN_WARPS);  // the drain warps of every CTA of the tile
        }
        mbar_init(mma_done, 1);
        mbar_init(&merge[0], 32 * DRAIN_WARPS);  // every lane: each releases its own staging stores
        mbar_init(&merge[1], 32 * DRAIN_WARPS);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        G::alloc(tmem_slot, TMEM_COLS);
        G::relinquish();
    }
    if (warp == PRODUCER_WARP && lane == 0) {
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        if (!Q6) {
            tma_prefetch_desc(&tmWs);
            tma_prefetch_desc(&tmXs);
        }
        if (C::SROWS > 0 && p.tma_store) tma_prefetch_desc(&tmY);
        tma_prefetch_desc(&tmD);
        tma_prefetch_desc(&tmDx);
        if (Q5) tma_prefetch_desc(&tmDm);
    }
    // barriers initialised and TMEM allocated in both CTAs before any cross-CTA traffic
    tc_fence_before();
    G::sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int64_t mt_count = (p.M + TMP - 1) / TMP;
    const int64_t nt_count = (p.N + CG * TN - 1) / (CG * TN);
    const int64_t tiles = mt_count * nt_count;
    const int64_t pair = CG == 2 ? (int64_t)cluster_id_x() : (int64_t)blockIdx.x;
    const int64_t pairs = CG == 2 ? (int64_t)cluster_count_x() : (int64_t)gridDim.x;
    const int64_t nb = p.K / kQKK;  // super-blocks
    const int64_t nchunks = (p.K + BK - 1) / BK;
    uint32_t* status = p.status;

    if (warp >= 8) {
        regs_dec<C::PRODUCER_REGS>();
        if (warp == PRODUCER_WARP && lane == 0) {
            // the even CTA's stage and min barriers, as cluster addresses
            const uint32_t full0 = CG == 2 ? cluster_map(smem_u32(full), 0) : 0u;
            const uint32_t mfull0 = CG == 2 ? cluster_map(smem_u32(mfull), 0) : 0u;
            int stage = 0, se = 0, me = 0;
            uint32_t ph = 0, sph = 0, mph = 0;
            for (int64_t tile = pair; tile < tiles; tile += pairs) {
                const int32_t m0 = (int32_t)((tile % mt_count) * TMP);
                const int32_t mc = m0 + (int32_t)(rank * XR);
                const int32_t nc = (int32_t)(p.n_first + (tile / mt_count) * CG * TN + rank * TN);
                for (int64_t kc = 0; kc < nchunks; kc++) {
                    if (kc % 4 == 0) {
                        const int32_t sb = (int32_t)(kc / 4);
                        // this CTA's scales for its drain
                        if (!mbar_wait(&sempty[se], sph ^ 1u, abort_flag, status, kDevTimeoutScaleEmpty)) goto done;
                        uint8_t* e = sb_region + se * C::SB_ENTRY;
                        mbar_expect_tx(&sfull[se], (Q5 ? 2 * 512 : 512) + TMP * 4);
                        tma_load_2d(e + C::OFF_DW, &tmD, &sfull[se], nc, sb);
                        if (Q5) tma_load_2d(e + C::OFF_DMW, &tmDm, &sfull[se], nc, sb);
                        tma_load_2d(e + C::OFF_DX, &tmDx, &sfull[se], m0, sb);
                        if (++se == C::SB_DEPTH) {
                            se = 0;
                            sph ^= 1u;
                        }
                        if (Q5) {
                            // this CTA's halves of the min-term operands
                            if (!mbar_wait(&mempty[me], mph ^ 1u, abort_flag, status, kDevTimeoutScaleEmpty)) goto done;
                            uint8_t* mn = min_region + me * C::MIN_ENTRY;
                            if (leader) mbar_expect_tx(&mfull[me], CG * C::MIN_ENTRY);
                            G::load(mn, &tmWs, &mfull[me], mfull0 + 8u * me, sb * 16, nc);
                            G::load(mn + SW32_W, &tmXs, &mfull[me], mfull0 + 8u * me, sb * 16, mc);
                            if (++me == DEPTH) {
                                me = 0;
                                mph ^= 1u;
                            }
                        }
                    }
                    if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, status, kDevTimeoutEmpty)) goto done;
                    uint8_t* st = smem + stage * C::STAGE;
                    const uint32_t fb = full0 + 8u * stage;
                    uint64_t* fl = &full[stage];
                    const int32_t kx = (int32_t)(kc * BK);
                    if (Q6) {
                        // chunk kc's even and parity planes sit side by side in the [N][2K] operand
                        if (leader) mbar_expect_tx(fl, CG * (2 * W_BYTES + C::X_BYTES));
                        G::load(st, &tmW, fl, fb, 2 * kx, nc);
                        G::load(st + W_BYTES, &tmW, fl, fb, 2 * kx + BK, nc);
                        G::load(st + 2 * W_BYTES, &tmX, fl, fb, kx, mc);
                    } else {
                        if (leader) mbar_expect_tx(fl, CG * (W_BYTES + C::X_BYTES));
                        G::load(st, &tmW, fl, fb, kx, nc);
                        G::load(st + W_BYTES, &tmX, fl, fb, kx, mc);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        } else if (warp == MMA_WARP && lane == 0 && leader) {
            int stage = 0, me = 0;
            uint32_t ph = 0, mph = 0;
            uint64_t gsb = 0;   // super-blocks issued: selects the slots' roles
            uint64_t item = 0;  // items issued (K-quant block-dot dump: every item in the next slot)
            for (int64_t tile = pair; tile < tiles; tile += pairs) {
                for (int64_t kc = 0; kc < nchunks; kc++) {
                    const int q = (int)(kc % 4);
                    if (Q5 && DUMP && q == 0) {
                        // dump: the min item first, in its own slot
                        if (!mbar_wait(&mfull[me], mph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                        const int s = (int)(item & 1);
                        if (!mbar_wait_cluster(&tempty[s], (uint32_t)((item >> 1) & 1) ^ 1u, abort_flag, status,
                                               kDevTimeoutTmemEmpty)) goto done;
                        tc_fence_after();
                        const uint32_t mn = smem_u32(min_region + me * C::MIN_ENTRY);
                        G::mma(tmem_base + (uint32_t)(s * TMP), desc_sw32(mn), desc_sw32(mn + SW32_W), IDESC, 0u);
                        G::commit(&tfull[s]);
                        G::commit(&mempty[me]);
                        item++;
                        if (++me == DEPTH) {
                            me = 0;
                            mph ^= 1u;
                        }
                    }
                    if (!mbar_wait(&full[stage], ph, abort_flag, status, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(smem + stage * C::STAGE);
                    const uint32_t x_addr = w_addr + (Q6 ? 2 * W_BYTES : W_BYTES);
                    {
                        // this stage's chunk: into the super-block's chunk slot (or, dumping, its own slot)
                        const bool first = DUMP || q == 0;
                        const bool last = DUMP || q == 3 || kc == nchunks - 1;
                        // slot and phase: Q5_K uses both slots once per super-block (phase
                        // gsb & 1); Q6_K and the dump use one slot per item, alternating
                        const uint64_t use = DUMP ? item : gsb;
                        const int cs = (int)(use & 1);
                        const uint32_t cpar = (Q5 && !DUMP) ? (uint32_t)(gsb & 1) : (uint32_t)((use >> 1) & 1);
                        if (first) {
                            if (!mbar_wait_cluster(&tempty[cs], cpar ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            tc_fence_after();
                        }
                        const uint32_t d = tmem_base + (uint32_t)(cs * TMP);
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const uint32_t koff = (uint32_t)k * 32u;
                            G::mma(d, desc_sw128(w_addr + koff), desc_sw128(x_addr + koff), IDESC,
                                         (first && k == 0) ? 0u : 1u);
                            if (Q6) G::mma(d, desc_sw128(w_addr + W_BYTES + koff), desc_sw128(x_addr + koff), IDESC, 1u);
                        }
                        if (Q5 && !DUMP && q == 2) {
                            // the min item, into the other slot: that slot held the previous
                            // super-block's chunk sum, whose drain overlapped the first three
                            // stages; the drain reads the min item during the last one
                            if (!mbar_wait(&mfull[me], mph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                            if (!mbar_wait_cluster(&tempty[cs ^ 1], cpar ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty))
                                goto done;
                            tc_fence_after();
                            const uint32_t mn = smem_u32(min_region + me * C::MIN_ENTRY);
                            G::mma(tmem_base + (uint32_t)((cs ^ 1) * TMP), desc_sw32(mn), desc_sw32(mn + SW32_W), IDESC, 0u);
                            G::commit(&tfull[cs ^ 1]);
                            G::commit(&mempty[me]);
                            if (++me == DEPTH) {
                                me = 0;
                                mph ^= 1u;
                            }
                        }
                        if (last) {
                            G::commit(&tfull[cs]);
                            if (DUMP)
                                item++;
                            else
                                gsb++;
                        }
                    }
                    G::commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------ drain warps --
        regs_inc<C::DRAIN_REGS>();
        const uint32_t quad = warp & 3u, half = warp >> 2;
        const uint32_t wrow = quad * 32u + lane;              // CTA-local weight row == TMEM lane
        const uint32_t lane_base = (quad * 32u) << 16;
        // slot releases go to the even CTA's barriers
        const uint32_t tempty0 = CG == 2 ? cluster_map(smem_u32(tempty), 0) : 0u;
        auto release = [&](int s) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader)
                    mbar_arrive(&tempty[s]);
                else
                    mbar_arrive_remote(tempty0 + 8u * (uint32_t)s);
            }
        };
        int se = 0;
        uint32_t sph = 0, mgph = 0;
        uint64_t gsb = 0, item = 0;
        // all drain warps meet (bounded wait, like every wait of this kernel)
        auto drain_meet = [&](int i) -> bool {
            mbar_arrive(&merge[i]);  // all lanes: a single lane's release does not cover the others' stores
            return mbar_wait(&merge[i], mgph, abort_flag, status, kDevTimeoutTmemFull);
        };
        for (int64_t tile = pair; tile < tiles; tile += pairs) {
            const int64_t m0 = (tile % mt_count) * TMP;
            const int64_t n0 = (tile / mt_count) * CG * TN + rank * TN;  // view-local, this CTA's rows
            const int64_t n = n0 + wrow;
            const int64_t mfirst = m0 + half * HC;
            float acc[HC];
#pragma unroll
            for (int i = 0; i < HC; i++) acc[i] = 0.f;
            {
                for (int64_t sb = 0; sb < nb; sb++) {
                    if (!mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                    const uint8_t* e = sb_region + se * C::SB_ENTRY;
                    const float* dx = reinterpret_cast<const float*>(e + C::OFF_DX) + half * HC;
                    if (!DUMP) {
                        const int cs = (int)(gsb & 1);
                        const uint32_t par = Q5 ? (uint32_t)(gsb & 1) : (uint32_t)((gsb >> 1) & 1);
                        // this thread's lanes: 32*quad + 16lh + 8h + lane/4
                        const float* dwv = reinterpret_cast<const float*>(e + C::OFF_DW) + quad * 32u + (lane >> 2);
                        if (Q5) {
                            // pix_dot_q5_K: summs += (-y.d * fp16(x.dmin)) * float(sum_j m_j * bsum_j)
                            const float* dmv = reinterpret_cast<const float*>(e + C::OFF_DMW) + quad * 32u + (lane >> 2);
                            const float4 w = make_float4(-dmv[0], -dmv[8], -dmv[16], -dmv[24]);
                            if (!mbar_wait(&tfull[cs ^ 1], par, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                            tc_fence_after();
                            drain_split(acc, tmem_base + lane_base + (uint32_t)((cs ^ 1) * TMP) + half * HC, dx, w, lane);
                            release(cs ^ 1);
                        }
                        // acc += (y.d * fp16(x.d)) * float(sumi)
                        const float4 w = make_float4(dwv[0], dwv[8], dwv[16], dwv[24]);
                        if (!mbar_wait(&tfull[cs], par, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                        tc_fence_after();
                        drain_split(acc, tmem_base + lane_base + (uint32_t)(cs * TMP) + half * HC, dx, w, lane);
                        release(cs);
                        gsb++;
                    } else {
                        // items in issue order: Q5_K the min sum, then the four chunk sums
                        constexpr int ITEMS = Q5 ? 5 : 4;
#pragma unroll 1
                        for (int it = 0; it < ITEMS; it++) {
                            const int s = (int)(item & 1);
                            if (!mbar_wait(&tfull[s], (uint32_t)((item >> 1) & 1), abort_flag, status, kDevTimeoutTmemFull))
                                goto done;
                            tc_fence_after();
                            const int64_t idx = Q5 ? sb * 5 + (it == 0 ? 4 : it - 1) : sb * 4 + it;
                            drain_dump<HC>(tmem_base + lane_base + (uint32_t)(s * TMP) + half * HC, p, idx, mfirst, n);
                            release(s);
                            item++;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sempty[se]);
                    if (++se == C::SB_DEPTH) {
                        se = 0;
                        sph ^= 1u;
                    }
                }
            }
            if (!DUMP && p.gated) {
                // gated weight: this CTA's lanes 64..127 hold the up projection of the
                // outputs whose gate projection lanes 0..63 hold (the repack interleaves
                // 64-row groups); the up warps hand their sums over through the staging
                // buffer and the gate warps finish tensor_silu + tensor_gate
                // (src/tensor.cpp:199-208, :334-345)
                float* xfer = reinterpret_cast<float*>(smem + off_staging<TYPE>()) + ((quad & 1) * 2 + half) * (HC * 32);
                if (!drain_meet(0)) goto done;  // the previous tile's hand-over has been read
                if (quad >= 2) {
#pragma unroll
                    for (int i = 0; i < HC; i++) xfer[i * 32 + lane] = acc[i];
                }
                if (!drain_meet(1)) goto done;
                mgph ^= 1u;
                if (quad < 2) {
#pragma unroll
                    for (int i = 0; i < HC; i++) {
                        // element i's output row (lane) and activation row (column)
                        const int c = i & 1, h = (i >> 1) & 1, k = (i >> 2) & 7, lh = (i >> 5) & 1, ch = i >> 6;
                        const int lo = 16 * lh + 8 * h + (int)(lane >> 2);
                        const int col = 64 * ch + 8 * k + 2 * (int)(lane & 3) + c;
                        const int64_t on = n0 / 2 + quad * 32 + lo, m = mfirst + col;
                        const float g = acc[i], u = xfer[i * 32 + lane];
                        if (on < p.N / 2 && m < p.M) p.y[m * p.ldy + on] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                    }
                }
            } else if (!DUMP) {
                // this thread's lanes (weight rows, CTA-local): 16lh + 8h + lane/4
                float bv[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int64_t nn = n0 + quad * 32 + 8 * i + (lane >> 2);
                    bv[i] = (p.bias && nn < p.N) ? p.bias[nn] : 0.f;
                }
                if (C::SROWS > 0 && p.tma_store) {
                    // each warp stages [SROWS activation rows][32 weight rows] blocks and
                    // stores each with one TMA store; lane 0 first waits until the warp's
                    // previous store has finished reading the buffer (no cross-warp sync)
                    constexpr int SR = C::SROWS > 0 ? C::SROWS : 64;
                    static_assert(SR == 64, "the 16x256b layout stages 64 columns per round");
                    float* stg = reinterpret_cast<float*>(smem + off_staging<TYPE>()) + warp * (SR * 32);
#pragma unroll
                    for (int r = 0; r < HC / SR; r++) {
                        if (lane == 0) bulk_wait_read_all();
                        __syncwarp();
#pragma unroll
                        for (int lh = 0; lh < 2; lh++)
#pragma unroll
                            for (int k = 0; k < 8; k++)
#pragma unroll
                                for (int h = 0; h < 2; h++)
#pragma unroll
                                    for (int c = 0; c < 2; c++) {
                                        const float v = acc[split_idx(r, lh, k, h, c)];
                                        stg[(8 * k + 2 * (lane & 3) + c) * 32 + 16 * lh + 8 * h + (lane >> 2)] =
                                            p.bias ? __fadd_rn(v, bv[2 * lh + h]) : v;
                                    }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmY, stg, (int32_t)(n0 + quad * 32), (int32_t)(mfirst + SR * r));
                            bulk_commit();
                        }
                        if (p.ndst && p.dst_vec4) {
                            // the peers' copies from the same staged block, 4 floats a lane:
                            // 8 lanes store one row's 128 contiguous bytes, a warp 4 rows
                            const int jr = lane >> 3, c4 = 4 * (lane & 7);
                            const int64_t nn = n0 + quad * 32 + c4;
                            for (int j = jr; j < SR; j += 4) {
                                const int64_t m = mfirst + SR * r + j;
                                if (m >= p.M) break;
                                const float4 v = *reinterpret_cast<const float4*>(stg + j * 32 + c4);
                                const int64_t off = m * p.ldy + p.col_off + nn;
                                if (nn + 3 < p.N) {
                                    for (int k = 0; k < p.ndst; k++) *reinterpret_cast<float4*>(p.ydst[k] + off) = v;
                                } else {
                                    const float vs[4] = {v.x, v.y, v.z, v.w};
                                    for (int q = 0; q < 4 && nn + q < p.N; q++)
                                        for (int k = 0; k < p.ndst; k++) p.ydst[k][off + q] = vs[q];
                                }
                            }
                        } else if (p.ndst) {
                            // the same, one float a lane: 32 lanes store 128 contiguous bytes
                            const int64_t nn = n0 + quad * 32 + lane;
                            if (nn < p.N) {
                                for (int j = 0; j < SR; j++) {
                                    const int64_t m = mfirst + SR * r + j;
                                    if (m >= p.M) break;
                                    const float v = stg[j * 32 + lane];
                                    const int64_t off = m * p.ldy + p.col_off + nn;
                                    for (int k = 0; k < p.ndst; k++) p.ydst[k][off] = v;
                                }
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int ch = 0; ch < 2; ch++)
#pragma unroll
                        for (int lh = 0; lh < 2; lh++)
#pragma unroll
                            for (int k = 0; k < 8; k++)
#pragma unroll
                                for (int h = 0; h < 2; h++)
#pragma unroll
                                    for (int c = 0; c < 2; c++) {
                                        const int64_t nn = n0 + quad * 32 + 16 * lh + 8 * h + (lane >> 2);
                                        const int64_t m = mfirst + 64 * ch + 8 * k + 2 * (lane & 3) + c;
                                        const float v = acc[split_idx(ch, lh, k, h, c)];
                                        if (nn < p.N && m < p.M) put_y(p, m, nn, p.bias ? __fadd_rn(v, bv[2 * lh + h]) : v);
                                    }
                }
            }
        }
    }
done:
    // outstanding output stores must finish reading shared memory before exit
    if (C::SROWS > 0 && p.tma_store && warp < DRAIN_WARPS && lane == 0) bulk_wait_all();
    // peer stores are visible system-wide before the kernel ends (the
    // N-sharded path's barrier after the kernel then orders them for the peers)
    if (p.ndst && warp < DRAIN_WARPS) __threadfence_system();
    if (warp == MMA_WARP && lane == 0 && leader) {
        // no MMA of this pair may still be writing TMEM when it is freed (after a
        // normal run the drains have consumed every result; this covers aborts)
        G::commit_local(mma_done);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(mma_done, 0) && global_ns() - t0 < PXQ_WAIT_NS) {
        }
    }
    __syncwarp();
    // the peer CTA no longer touches this CTA's barriers or TMEM after this
    tc_fence_before();
    G::sync();
    tc_fence_after();
    if (warp == 0) G::dealloc(tmem_base, TMEM_COLS);
}

template <uint32_t TYPE, bool DUMP>
cudaError_t launch_typed(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    auto kern = k_gemm<TYPE, DUMP>;
    constexpr int smem = smem_bytes<TYPE>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    constexpr int CG = Cfg<TYPE>::CG;
    const int64_t tiles = ((op.M + Cfg<TYPE>::TMP - 1) / Cfg<TYPE>::TMP) * ((op.N + CG * TN - 1) / (CG * TN));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = CG == 2 ? 1 : 0;
    int64_t groups = num_sms;  // one CTA per SM
    if (CG == 2) {
        // pairs that can be resident at once
        static int max_pairs = 0;
        static std::once_flag once;
        std::call_once(once, [&] {
            cfg.gridDim = dim3(2 * (num_sms / 2));
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
                cudaGetLastError();
                n = num_sms / 2;
            }
            max_pairs = n;
        });
        groups = max_pairs;
    }
    if (tiles < groups) groups = tiles;
    if (groups < 1) groups = 1;
    cfg.gridDim = dim3((unsigned)(CG * groups));
    Params p{op.M, op.N, op.K, op.n_first, op.y, op.ldy, op.bias, op.dump, op.status, (op.tma_store && !DUMP) ? 1 : 0, op.gated,
             op.ndst, op.dst_vec4, op.col_off, {}};
    for (int k = 0; k < kMaxScatter; k++) p.ydst[k] = op.ydst[k];
    return cudaLaunchKernelEx(&cfg, kern, op.tm[0], op.tm[1], op.tm[2], op.tm[3], op.tm[4], op.tm[5], op.tm[6], op.tm_y, p);
}

}  // namespace

// Q8_0 (gemm_q8.cu): one CTA per 128 x 128 tile, 32-row stores
int gemm_activation_rows(uint32_t type) { return type == kTypeQ8_0 ? 128 : Cfg<kTypeQ5_K>::XR; }
int gemm_tile_activation_rows(uint32_t type) { return type == kTypeQ8_0 ? 128 : Cfg<kTypeQ5_K>::TMP; }
int gemm_store_rows(uint32_t type)
{
    return type == kTypeQ8_0 ? 32 : type == kTypeQ5_K ? Cfg<kTypeQ5_K>::SROWS : Cfg<kTypeQ6_K>::SROWS;
}

cudaError_t launch_gemm(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    if (op.type == kTypeQ8_0) return launch_gemm_q8(op, num_sms, s);
    if (op.type == kTypeQ5_K) {
        return op.dump ? launch_typed<kTypeQ5_K, true>(op, num_sms, s) : launch_typed<kTypeQ5_K, false>(op, num_sms, s);
    }
    if (op.type == kTypeQ6_K) {
        return op.dump ? launch_typed<kTypeQ6_K, true>(op, num_sms, s) : launch_typed<kTypeQ6_K, false>(op, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace pxq
