// gemm.cu -- large-M quantized GEMM on the 5th-generation tensor cores.
//
// Computes Y[m, n] = sum over K-blocks b of  s(m,n,b) * I(m,n,b)
// where I is the exact integer dot of one block of quants and s the product
// of the block scales -- the arithmetic of pix_dot_q8_0
// (src/kernels_quant.cpp:339-365) and pix_dot_q5_K (:163-254) as driven by
// cpu_quant_matmul (:389-400), for every (activation row m, weight row n).
//
// Design (sm_100a):
//   * Operands are exact fp16 copies of the int8 quants (activations from
//     quantize.cu, weights from the one-time repack in repack.cu).  A
//     kind::f16 tcgen05.mma with fp32 accumulation computes each block dot
//     exactly (|I| <= 32*127*127 for Q8_0, <= 64*127*1953 < 2^24 for a Q5_K
//     64-value chunk) and hands the drain a float.  (kind::i8 runs the MMA
//     twice as fast but needs an int->float conversion per element per block
//     on the CUDA cores, which bound this kernel.)
//   * Orientation: TMEM lanes are WEIGHT rows (the MMA's M side), TMEM
//     columns are ACTIVATION rows.  Per-weight-row scales are then per-thread
//     scalars, and the 32 lanes of a warp store 32 consecutive outputs.
//   * Q8_0: the per-block scale product dW[n,b]*dX[m,b] is itself computed by
//     the tensor core -- a K=16 MMA of a one-hot weight-scale tile (dW at
//     position b%16) against the activations' 16-block fp16 scale tile, exact
//     because fp16*fp16 fits fp32 -- so the drain is one FMA per element per
//     block and reads no scale from shared memory.
//   * Q5_K: 6-bit sub-block scales are folded into the weight operand
//     (sc*q5 <= 1953, exact in fp16), so every 64-value chunk dot is exact in
//     the fp32 accumulator, and the four chunks of a super-block, which share
//     its scale dW*dX, accumulate into one TMEM slot: one drain per
//     super-block.  Their sum is exact while it stays below 2^24 in magnitude
//     (always, for real activations; the reference rounds its int32 sum to
//     fp32 once, the tensor core at most at each chunk boundary beyond that).
//     The block-dot dump (pxq_gemm_block_dots) drains every chunk on its own,
//     so the exact int32 chunk dots stay checkable.  The min term
//     sum_j m_j*bsum_j is a K=16 MMA per super-block on exact (hi, lo) splits,
//     drained first.
//   * Q6_K (pix_dot_q6_K, :256-337): the 8-bit scale and the -32 offset fold
//     into v = sc*(q6-32), |v| <= 4096 -- 13 bits, one more than fp16 holds
//     for odd values.  The repack splits v into an even part (exact in fp16)
//     and its parity bit, two operand planes that two MMAs per K step
//     accumulate into the same TMEM slot, so the chunk dots stay exact
//     integers.  No min term; one drain per super-block.
//   * Warp roles (12 warps, 3 warpgroups): warpgroups 0-1 drain TMEM (warp w
//     reads lane quadrant w%4 and column half w/4) with 232 registers
//     (setmaxnreg); warpgroup 2 runs the TMA producer (warp 8) and the
//     single-thread MMA issuer (warp 9) with 40.  Persistent CTAs walk
//     128x128 output tiles; four 128-column TMEM slots let the MMA run up to
//     four items ahead of the drain.
//   * Every mbarrier wait is bounded (pxq_device.cuh).  Every CTA loads its
//     own tiles from this GPU's HBM; no cluster broadcast of any kind.
#include <cuda.h>
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int TN = 128;                // weight rows per tile (TMEM lanes, MMA M)
constexpr int TM = 128;                // activation rows per tile (TMEM columns, MMA N)
constexpr int BK = 64;                 // fp16 K elements per stage (128-byte rows)
constexpr int W_BYTES = TN * BK * 2;   // 16 KB
constexpr int X_BYTES = TM * BK * 2;   // 16 KB
constexpr int SW32_TILE = 128 * 32;    // [128][16] fp16 tile, 32-byte swizzle: 4 KB
constexpr int DRAIN_WARPS = 8;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int THREADS = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr int SLOTS = 4;               // TMEM slots of 128 columns
constexpr int MAX_STAGES = 6;
constexpr uint32_t IDESC = idesc_f16_f32(TN, TM);

// output staging for the TMA-store epilogue: per drain warp [64 activation rows][32 weight rows] fp32
constexpr int STAGING = 2 * 64 * TN * 4;                                  // 64 KB
// Q8_0 stage: W | X | one-hot weight scales for the stage's 2 blocks | activation scales (16 blocks)
constexpr int Q80_STAGES = 3;
constexpr int Q80_STAGE = W_BYTES + X_BYTES + 2 * SW32_TILE + SW32_TILE;  // 44 KB
// Q5_K stage: W | X;  super-block entries: Wmin | Xmin | dW | dminW | dX
constexpr int Q5_STAGES = 4;
constexpr int Q5_STAGE = W_BYTES + X_BYTES;                                // 32 KB
constexpr int Q5_SB_ENTRY = 2 * SW32_TILE + 3 * 512;                      // 9.5 KB
constexpr int Q5_SB_DEPTH = 2;
// Q6_K stage: W even part | W parity part | X;  super-block entries: dW | dX
constexpr int Q6_STAGES = 3;
constexpr int Q6_STAGE = 2 * W_BYTES + X_BYTES;                            // 48 KB
constexpr int Q6_SB_ENTRY = 2 * 512;

template <uint32_t TYPE>
struct Cfg;
template <>
struct Cfg<kTypeQ8_0> {
    static constexpr int STAGES = Q80_STAGES;
    static constexpr int STAGE = Q80_STAGE;
    static constexpr int SB_ENTRY = 0;
    static constexpr int SB_REGION = 0;
    static constexpr int OFF_DW = 0, OFF_DMW = 0, OFF_DX = 0;  // no super-block entries
};
template <>
struct Cfg<kTypeQ5_K> {
    static constexpr int STAGES = Q5_STAGES;
    static constexpr int STAGE = Q5_STAGE;
    static constexpr int SB_ENTRY = Q5_SB_ENTRY;
    static constexpr int SB_REGION = Q5_SB_ENTRY * Q5_SB_DEPTH;
    static constexpr int OFF_DW = 2 * SW32_TILE, OFF_DMW = OFF_DW + 512, OFF_DX = OFF_DW + 1024;  // in an entry
};
template <>
struct Cfg<kTypeQ6_K> {
    static constexpr int STAGES = Q6_STAGES;
    static constexpr int STAGE = Q6_STAGE;
    static constexpr int SB_ENTRY = Q6_SB_ENTRY;
    static constexpr int SB_REGION = Q6_SB_ENTRY * Q5_SB_DEPTH;
    static constexpr int OFF_DW = 0, OFF_DMW = 0, OFF_DX = 512;
};

template <uint32_t TYPE>
__host__ __device__ constexpr int off_staging()
{
    return Cfg<TYPE>::STAGES * Cfg<TYPE>::STAGE + Cfg<TYPE>::SB_REGION;
}
template <uint32_t TYPE>
__host__ __device__ constexpr int off_bar()
{
    return off_staging<TYPE>() + STAGING;
}
constexpr int NUM_BARS = 2 * MAX_STAGES + 2 * Q5_SB_DEPTH + 2 * SLOTS;  // full/empty, sfull/sempty, tfull/tempty
template <uint32_t TYPE>
__host__ __device__ constexpr int smem_bytes()
{
    return off_bar<TYPE>() + NUM_BARS * 8 + 16 + 1024;
}
static_assert(Q80_STAGES <= MAX_STAGES && Q5_STAGES <= MAX_STAGES && Q6_STAGES <= MAX_STAGES, "stage count");
static_assert(smem_bytes<kTypeQ8_0>() <= 232448, "Q8_0 shared memory");
static_assert(smem_bytes<kTypeQ5_K>() <= 232448, "Q5_K shared memory");
static_assert(smem_bytes<kTypeQ6_K>() <= 232448, "Q6_K shared memory");
static_assert(Q6_STAGE % 1024 == 0 && Q5_STAGE % 1024 == 0, "128B-swizzled tiles need 1024-byte alignment");

struct Params {
    int64_t M, N, K;
    int64_t n_first;
    float* y;
    int64_t ldy;
    const float* bias;
    float* dump;
    uint32_t* status;
    int tma_store;  // 1: epilogue through shared memory + TMA store (tmY)
};

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }
__device__ __forceinline__ uint64_t desc_sw32(uint32_t saddr) { return smem_desc(saddr, 16, 256, 6); }

// tensor maps:
//   tmW   weight operand fp16 [N][K] (Q6_K: [N][2K])  box {64, 128}  128B swizzle
//   tmX   activation operand fp16 [M][K]        box {64, 128}  128B swizzle
//   Q8_0: tmWs  one-hot weight scales fp16 [N][nb*16]   box {16, 128} 32B swizzle
//         tmXs  activation scales fp16 [M][nb]          box {16, 128} 32B swizzle
//   Q5_K: tmWs  weight min operand fp16 [N][nsb*16]     box {16, 128} 32B swizzle
//         tmXs  activation min operand fp16 [M][nsb*16] box {16, 128} 32B swizzle
//         tmD   weight d   fp32 [nsb][N4]  box {128, 1}
//         tmDm  weight dmin fp32 [nsb][N4] box {128, 1}
//         tmDx  activation d fp32 [nsb][M4] box {128, 1}
//   Q6_K: tmD, tmDx as for Q5_K (the others unused)
template <uint32_t TYPE, bool DUMP>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
           const __grid_constant__ CUtensorMap tmWs, const __grid_constant__ CUtensorMap tmXs,
           const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmDm,
           const __grid_constant__ CUtensorMap tmDx, const __grid_constant__ CUtensorMap tmY, const Params p)
{
    using C = Cfg<TYPE>;
    constexpr bool Q8 = TYPE == kTypeQ8_0;
    constexpr bool Q6 = TYPE == kTypeQ6_K;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + off_bar<TYPE>());
    uint64_t* full = bars;
    uint64_t* empty = bars + MAX_STAGES;
    uint64_t* sfull = bars + 2 * MAX_STAGES;
    uint64_t* sempty = sfull + Q5_SB_DEPTH;
    uint64_t* tfull = sempty + Q5_SB_DEPTH;
    uint64_t* tempty = tfull + SLOTS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    uint8_t* sb_region = smem + STAGES * C::STAGE;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < Q5_SB_DEPTH; i++) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sempty[i], Q6 ? DRAIN_WARPS : DRAIN_WARPS + 1);  // drain warps (+ the MMA thread: Q5_K min operands)
        }
        for (int i = 0; i < SLOTS; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], DRAIN_WARPS);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == PRODUCER_WARP && lane == 0) {
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmWs);
        tma_prefetch_desc(&tmXs);
        if (p.tma_store) tma_prefetch_desc(&tmY);
        if (!Q8) {
            tma_prefetch_desc(&tmD);
            tma_prefetch_desc(&tmDm);
            tma_prefetch_desc(&tmDx);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int64_t mt_count = (p.M + TM - 1) / TM;
    const int64_t nt_count = (p.N + TN - 1) / TN;
    const int64_t tiles = mt_count * nt_count;
    const int64_t nb = Q8 ? p.K / kQK8_0 : p.K / kQKK;  // blocks (Q8_0) or super-blocks (Q5_K)
    const int64_t nchunks = (p.K + BK - 1) / BK;
    uint32_t* status = p.status;

    if (warp >= 8) {
        regs_dec<40>();
        if (warp == PRODUCER_WARP && lane == 0) {
            int stage = 0;
            uint32_t ph = 0;
            int se = 0;
            uint32_t sph = 0;
            for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                const int32_t m0 = (int32_t)((tile % mt_count) * TM);
                const int32_t n0 = (int32_t)(p.n_first + (tile / mt_count) * TN);
                for (int64_t kc = 0; kc < nchunks; kc++) {
                    if (!Q8 && kc % 4 == 0) {
                        if (!mbar_wait(&sempty[se], sph ^ 1u, abort_flag, status, kDevTimeoutScaleEmpty)) goto done;
                        uint8_t* e = sb_region + se * Cfg<TYPE>::SB_ENTRY;
                        const int32_t sb = (int32_t)(kc / 4);
                        mbar_expect_tx(&sfull[se], Cfg<TYPE>::SB_ENTRY);
                        if (!Q6) {
                            tma_load_2d(e, &tmWs, &sfull[se], sb * 16, n0);
                            tma_load_2d(e + SW32_TILE, &tmXs, &sfull[se], sb * 16, m0);
                            tma_load_2d(e + C::OFF_DMW, &tmDm, &sfull[se], n0, sb);
                        }
                        tma_load_2d(e + C::OFF_DW, &tmD, &sfull[se], n0, sb);
                        tma_load_2d(e + C::OFF_DX, &tmDx, &sfull[se], m0, sb);
                        if (++se == Q5_SB_DEPTH) {
                            se = 0;
                            sph ^= 1u;
                        }
                    }
                    if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, status, kDevTimeoutEmpty)) goto done;
                    uint8_t* st = smem + stage * C::STAGE;
                    if (Q8) {
                        const int nblk = (2 * kc + 1 < nb) ? 2 : 1;
                        mbar_expect_tx(&full[stage], W_BYTES + X_BYTES + (nblk + 1) * SW32_TILE);
                        tma_load_2d(st, &tmW, &full[stage], (int32_t)(kc * BK), n0);
                        tma_load_2d(st + W_BYTES, &tmX, &full[stage], (int32_t)(kc * BK), m0);
                        for (int b = 0; b < nblk; b++)
                            tma_load_2d(st + W_BYTES + X_BYTES + b * SW32_TILE, &tmWs, &full[stage],
                                        (int32_t)((2 * kc + b) * 16), n0);
                        tma_load_2d(st + W_BYTES + X_BYTES + 2 * SW32_TILE, &tmXs, &full[stage],
                                    (int32_t)(((2 * kc) / 16) * 16), m0);
                    } else if (Q6) {
                        // chunk kc's even and parity planes sit side by side in the [N][2K] operand
                        mbar_expect_tx(&full[stage], 2 * W_BYTES + X_BYTES);
                        tma_load_2d(st, &tmW, &full[stage], (int32_t)(kc * 2 * BK), n0);
                        tma_load_2d(st + W_BYTES, &tmW, &full[stage], (int32_t)(kc * 2 * BK + BK), n0);
                        tma_load_2d(st + 2 * W_BYTES, &tmX, &full[stage], (int32_t)(kc * BK), m0);
                    } else {
                        mbar_expect_tx(&full[stage], W_BYTES + X_BYTES);
                        tma_load_2d(st, &tmW, &full[stage], (int32_t)(kc * BK), n0);
                        tma_load_2d(st + W_BYTES, &tmX, &full[stage], (int32_t)(kc * BK), m0);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        } else if (warp == MMA_WARP && lane == 0) {
            int stage = 0;
            uint32_t ph = 0;
            int slot = 0;
            uint32_t tph = 0;
            int se = 0;
            uint32_t sph = 0;
            for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                for (int64_t kc = 0; kc < nchunks; kc++) {
                    if (!Q8 && !Q6 && kc % 4 == 0) {
                        // min-term item of this super-block, drained first
                        if (!mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                        if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                        tc_fence_after();
                        const uint32_t e = smem_u32(sb_region + se * Q5_SB_ENTRY);
                        mma_f16(tmem_base + (uint32_t)slot * TM, desc_sw32(e), desc_sw32(e + SW32_TILE), IDESC, 0u);
                        mma_commit(&tfull[slot]);
                        mma_commit(&sempty[se]);
                        if (++slot == SLOTS) {
                            slot = 0;
                            tph ^= 1u;
                        }
                        if (++se == Q5_SB_DEPTH) {
                            se = 0;
                            sph ^= 1u;
                        }
                    }
                    if (!mbar_wait(&full[stage], ph, abort_flag, status, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(smem + stage * C::STAGE);
                    const uint32_t x_addr = w_addr + (Q6 ? 2 * W_BYTES : W_BYTES);
                    if (Q8) {
                        const uint32_t ws_addr = x_addr + X_BYTES;
                        const uint32_t xs_addr = ws_addr + 2 * SW32_TILE;
#pragma unroll
                        for (int blk = 0; blk < 2; blk++) {
                            if (2 * kc + blk >= nb) break;
                            // slots (slot, slot+1) hold (scale product, block dot); slot is even
                            if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            if (!mbar_wait(&tempty[slot + 1], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            tc_fence_after();
                            const uint32_t ds = tmem_base + (uint32_t)slot * TM;
                            // the activation scale tile covers blocks 16*g .. 16*g+15; the one-hot
                            // weight tile selects block (2kc+blk) % 16 of it
                            mma_f16(ds, desc_sw32(ws_addr + blk * SW32_TILE), desc_sw32(xs_addr), IDESC, 0u);
#pragma unroll
                            for (int k = 0; k < 2; k++) {
                                const uint32_t koff = (uint32_t)(blk * 2 + k) * 32u;  // 16 fp16 = 32 bytes
                                mma_f16(ds + TM, desc_sw128(w_addr + koff), desc_sw128(x_addr + koff), IDESC, (uint32_t)k);
                            }
                            mma_commit(&tfull[slot]);
                            slot += 2;
                            if (slot == SLOTS) {
                                slot = 0;
                                tph ^= 1u;
                            }
                        }
                    } else {
                        // K-quants: the four 64-value chunks of a super-block share its scale,
                        // so they accumulate into one TMEM slot (one drain per super-block);
                        // the block-dot dump keeps one slot per chunk.  Q6_K adds each K step's
                        // parity plane into the same accumulator.
                        const bool first = DUMP || kc % 4 == 0;
                        const bool last = DUMP || kc % 4 == 3 || kc == nchunks - 1;
                        if (first) {
                            if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            tc_fence_after();
                        }
                        const uint32_t d = tmem_base + (uint32_t)slot * TM;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const uint32_t koff = (uint32_t)k * 32u;
                            mma_f16(d, desc_sw128(w_addr + koff), desc_sw128(x_addr + koff), IDESC,
                                    (first && k == 0) ? 0u : 1u);
                            if (Q6) mma_f16(d, desc_sw128(w_addr + W_BYTES + koff), desc_sw128(x_addr + koff), IDESC, 1u);
                        }
                        if (last) {
                            mma_commit(&tfull[slot]);
                            if (++slot == SLOTS) {
                                slot = 0;
                                tph ^= 1u;
                            }
                        }
                    }
                    mma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------ drain warps --
        regs_inc<232>();
        const uint32_t quad = warp & 3u, half = warp >> 2;
        const uint32_t wrow = quad * 32u + lane;              // tile-local weight row == TMEM lane
        const uint32_t lane_base = (quad * 32u) << 16;
        int slot = 0;
        uint32_t tph = 0;
        int se = 0;
        uint32_t sph = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int64_t m0 = (tile % mt_count) * TM;
            const int64_t n0 = (tile / mt_count) * TN;  // view-local
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; i++) acc[i] = 0.f;
            if (Q8) {
                for (int64_t b = 0; b < nb; b++) {
                    if (!mbar_wait(&tfull[slot], tph, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                    tc_fence_after();
                    const uint32_t ts = tmem_base + lane_base + (uint32_t)slot * TM + half * 64u;
                    uint32_t sv[32], sv2[32], iv[32], iv2[32];
                    tmem_ld32(ts, sv);
                    tmem_ld32(ts + 32, sv2);
                    tmem_ld32(ts + TM, iv);
                    tmem_ld32(ts + TM + 32, iv2);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&tempty[slot]);
                        mbar_arrive(&tempty[slot + 1]);
                    }
                    if (DUMP) {
                        const int64_t n = n0 + wrow;
#pragma unroll
                        for (int j = 0; j < 64; j++) {
                            const int64_t m = m0 + half * 64 + j;
                            if (n < p.N && m < p.M)
                                p.dump[(b * p.M + m) * p.N + n] = __uint_as_float(j < 32 ? iv[j] : iv2[j - 32]);
                        }
                    } else {
                        // pix_dot_q8_0: acc = fma(fp16(dw)*fp16(dx), float(block dot), acc), two per instruction
#pragma unroll
                        for (int j = 0; j < 32; j += 2)
                            ffma2(acc[j], acc[j + 1], __uint_as_float(sv[j]), __uint_as_float(sv[j + 1]), __uint_as_float(iv[j]),
                                  __uint_as_float(iv[j + 1]));
#pragma unroll
                        for (int j = 0; j < 32; j += 2)
                            ffma2(acc[32 + j], acc[33 + j], __uint_as_float(sv2[j]), __uint_as_float(sv2[j + 1]),
                                  __uint_as_float(iv2[j]), __uint_as_float(iv2[j + 1]));
                    }
                    slot += 2;
                    if (slot == SLOTS) {
                        slot = 0;
                        tph ^= 1u;
                    }
                }
            } else {
                for (int64_t sb = 0; sb < nb; sb++) {
                    if (!mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                    const uint8_t* e = sb_region + se * C::SB_ENTRY;
                    const float dw = reinterpret_cast<const float*>(e + C::OFF_DW)[wrow];
                    const float4* dx4 = reinterpret_cast<const float4*>(e + C::OFF_DX) + half * 16;
                    float s[64];
                    if (Q6) {
                        // pix_dot_q6_K: d = y.d * fp16(x.d)
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const float4 v = dx4[j];
                            fmul2(s[4 * j + 0], s[4 * j + 1], v.x, v.y, dw, dw);
                            fmul2(s[4 * j + 2], s[4 * j + 3], v.z, v.w, dw, dw);
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sempty[se]);
                    } else {
                        // pix_dot_q5_K: dmin = -y.d * fp16(x.dmin)
                        const float dmw = reinterpret_cast<const float*>(e + C::OFF_DMW)[wrow];
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const float4 v = dx4[j];
                            fmul2(s[4 * j + 0], s[4 * j + 1], -v.x, -v.y, dmw, dmw);
                            fmul2(s[4 * j + 2], s[4 * j + 3], -v.z, -v.w, dmw, dmw);
                        }
                    }
                    // items: Q5_K the min term, then the super-block's chunk sum; Q6_K the
                    // chunk sum alone (one item per chunk when dumping block dots)
                    constexpr int ITEMS = Q6 ? (DUMP ? 4 : 1) : (DUMP ? 5 : 2);
#pragma unroll 1
                    for (int it = 0; it < ITEMS; it++) {
                        if (!Q6 && it == 1) {
                            // d = y.d * fp16(x.d), cached for the four chunks
#pragma unroll
                            for (int j = 0; j < 16; j++) {
                                const float4 v = dx4[j];
                                fmul2(s[4 * j + 0], s[4 * j + 1], v.x, v.y, dw, dw);
                                fmul2(s[4 * j + 2], s[4 * j + 3], v.z, v.w, dw, dw);
                            }
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&sempty[se]);
                        }
                        if (!mbar_wait(&tfull[slot], tph, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                        tc_fence_after();
                        const uint32_t ta = tmem_base + lane_base + (uint32_t)slot * TM + half * 64u;
                        uint32_t v0[32], v1[32];
                        tmem_ld32(ta, v0);
                        tmem_ld32(ta + 32, v1);
                        tmem_ld_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[slot]);
                        if (DUMP) {
                            const int64_t item = Q6 ? sb * 4 + it : sb * 5 + (it == 0 ? 4 : it - 1);
                            const int64_t n = n0 + wrow;
#pragma unroll
                            for (int j = 0; j < 64; j++) {
                                const int64_t m = m0 + half * 64 + j;
                                if (n < p.N && m < p.M)
                                    p.dump[(item * p.M + m) * p.N + n] = __uint_as_float(j < 32 ? v0[j] : v1[j - 32]);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; j += 2)
                                ffma2(acc[j], acc[j + 1], s[j], s[j + 1], __uint_as_float(v0[j]), __uint_as_float(v0[j + 1]));
#pragma unroll
                            for (int j = 0; j < 32; j += 2)
                                ffma2(acc[32 + j], acc[33 + j], s[32 + j], s[33 + j], __uint_as_float(v1[j]),
                                      __uint_as_float(v1[j + 1]));
                        }
                        if (++slot == SLOTS) {
                            slot = 0;
                            tph ^= 1u;
                        }
                    }
                    if (++se == Q5_SB_DEPTH) {
                        se = 0;
                        sph ^= 1u;
                    }
                }
            }
            if (!DUMP) {
                const int64_t n = n0 + wrow;
                const float bv = (p.bias && n < p.N) ? p.bias[n] : 0.f;
                if (p.tma_store) {
                    // each warp stages its [64 activation rows][32 weight rows] block and
                    // stores it with one TMA store; lane 0 first waits until the warp's
                    // previous store has finished reading the buffer (no cross-warp sync)
                    float* stg = reinterpret_cast<float*>(smem + off_staging<TYPE>()) + warp * (64 * 32);
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 64; j++) stg[j * 32 + lane] = p.bias ? __fadd_rn(acc[j], bv) : acc[j];
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmY, stg, (int32_t)(n0 + quad * 32), (int32_t)(m0 + half * 64));
                        bulk_commit();
                    }
                } else if (n < p.N) {
                    // lane = weight row: for each activation row, 32 lanes store 128 contiguous bytes
                    float* yc = p.y + n;
#pragma unroll
                    for (int j = 0; j < 64; j++) {
                        const int64_t m = m0 + half * 64 + j;
                        if (m < p.M) yc[m * p.ldy] = p.bias ? __fadd_rn(acc[j], bv) : acc[j];
                    }
                }
            }
        }
    }
done:
    // outstanding output stores must finish reading shared memory before exit
    if (p.tma_store && warp < DRAIN_WARPS && lane == 0) bulk_wait_all();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, TMEM_COLS);
}

template <uint32_t TYPE, bool DUMP>
cudaError_t launch_typed(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    auto kern = k_gemm<TYPE, DUMP>;
    constexpr int smem = smem_bytes<TYPE>();
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int64_t tiles = ((op.M + TM - 1) / TM) * ((op.N + TN - 1) / TN);
    int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid < 1) grid = 1;
    Params p{op.M, op.N, op.K, op.n_first, op.y, op.ldy, op.bias, op.dump, op.status, (op.tma_store && !DUMP) ? 1 : 0};
    kern<<<grid, THREADS, smem, s>>>(op.tm[0], op.tm[1], op.tm[2], op.tm[3], op.tm[4], op.tm[5], op.tm[6], op.tm_y, p);
    return cudaGetLastError();
}

}  // namespace

int gemm_smem_bytes() { return smem_bytes<kTypeQ8_0>(); }

cudaError_t launch_gemm(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    if (op.type == kTypeQ8_0) {
        return op.dump ? launch_typed<kTypeQ8_0, true>(op, num_sms, s) : launch_typed<kTypeQ8_0, false>(op, num_sms, s);
    }
    if (op.type == kTypeQ5_K) {
        return op.dump ? launch_typed<kTypeQ5_K, true>(op, num_sms, s) : launch_typed<kTypeQ5_K, false>(op, num_sms, s);
    }
    if (op.type == kTypeQ6_K) {
        return op.dump ? launch_typed<kTypeQ6_K, true>(op, num_sms, s) : launch_typed<kTypeQ6_K, false>(op, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace pxq
