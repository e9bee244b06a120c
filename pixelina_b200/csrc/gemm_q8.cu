// gemm_q8.cu -- large-M Q8_0 GEMM on the 5th-generation tensor cores.
//
// Computes, for every activation row m and weight row n,
//     Y[m, n] = sum over 32-blocks b of  (dW[n,b] * dX[m,b]) * I(m,n,b)
// where I is the exact integer dot of the block's int8 quants -- the
// arithmetic of pix_dot_q8_0 (src/kernels_quant.cpp:339-365: the fp32
// product of the two fp16 block scales times the float of an exact int32
// dot, accumulated in fp32) as driven by cpu_quant_matmul (:389-400).
//
// Design (sm_100a, one CTA per SM, persistent over 128 x 128 output tiles;
// drain warps plus one warpgroup for the producer and the MMA issuers):
//   * Per 32-block the tensor core computes the block dots I into TMEM and
//     the drain accumulates S * I per element.  Operand kinds
//     (GemmOperands::q8_kind, PXQ_Q8_0_MMA):
//       2 (default, fastest measured): exact fp16 copies of the quants, two
//         kind::f16 MMAs (K = 16 each) per block for the block dots I (exact
//         in fp32: |I| <= 32 * 127 * 127), and a K = 16 kind::f16 MMA of a
//         one-hot weight-scale tile against the activations' fp16 scale tile
//         for S = dW * dX, exact because fp16 x fp16 fits fp32
//         (k_gemm_q8s<., false, .>).  TMEM holds (S, I) for two blocks; the
//         drain does one packed FMA per element pair and block and reads no
//         scales from shared memory.  Eight drain warps of 64 columns each
//         (PXQ_Q8_0_DRAIN=16: sixteen of 32).
//       4: the same with the int8 quants and one kind::i8 MMA (K = 32) per
//         block for I (k_gemm_q8s<., true, .>): half the operand bytes and
//         one MMA fewer, but the drain converts every int32 dot to fp32.
//       0: fp16 copies, kind::f16 for I; the drain forms S = dW * dX itself
//         from fp32 block-major scale planes (k_gemm_q8s<., false, 8, true>):
//         a packed multiply and a packed FMA per element pair and block,
//         four blocks of I in TMEM.  Each drain warp reads its 64 activation
//         scales per block as shared-memory broadcasts, which set its speed.
//       1: as 0 with the int8 quants and kind::i8 MMAs plus an int -> float
//         conversion per element in the drain (k_gemm_q8s<., true, 8, true>).
//       3: kind 0's operands on CTA pairs (k_gemm_q8p, below).
//   * Scales for kinds 0 and 1 come by TMA into a ring of their own that the
//     drain releases, so an operand stage is free as soon as its MMAs are done.
//   * Tiles are walked in groups of 16 activation-row tiles, so the CTAs
//     running at the same time share their operand rows in L2.
//   * Every mbarrier wait is bounded (pxq_device.cuh); no TMA load uses a
//     cluster multicast, and every CTA loads from this GPU's memory only.
// The epilogue (bias, TMA-store staging, stores into peers' outputs for the
// N-sharded path, the gated feed-forward product, the block-dot dump) is
// the one of gemm.cu, per accumulator layout.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int Q8_TN = 128;           // weight rows per tile (TMEM lanes)
constexpr int Q8_TM = 128;           // activation rows per tile (TMEM columns per slot)
constexpr int Q8_OP_BYTES = 128 * 128;  // one operand per stage: 128 rows x one 128-byte swizzle row
constexpr int Q8_STAGE = 2 * Q8_OP_BYTES;
constexpr int Q8_GROUP_M = 16;       // activation-row tiles per raster group
constexpr int Q8_STAGING = 64 * 1024;  // output staging: every drain warp's [activation rows][32 weight rows] fp32

template <int OPK>
struct Q8Op;
template <>
struct Q8Op<0> {                     // fp16 operands, kind::f16
    static constexpr int BPS = 2;    // 32-blocks per stage (64 fp16 = 128 bytes)
    static constexpr int SD = 8;     // scale ring entries
};
template <>
struct Q8Op<1> {                     // int8 operands, kind::i8
    static constexpr int BPS = 4;    // 32-blocks per stage (128 int8 = 128 bytes)
    static constexpr int SD = 6;
};

template <int OPK>
__host__ __device__ constexpr int q8_entry_bytes() { return Q8Op<OPK>::BPS * 2 * 128 * 4; }  // dW | dX fp32
struct Q8Params {
    int64_t M, N, K;
    int64_t n_first;
    float* y;
    int64_t ldy;
    const float* bias;
    float* dump;
    uint32_t* status;
    int tma_store;
    int gated;
    int ndst;
    int dst_vec4;
    int64_t col_off;
    float* ydst[kMaxScatter];
    int tma_dst;  // the scatter as TMA stores through Q8PeerMaps (one-CTA kernels)
};

// Maps of the scatter destinations (ydst[k] + col_off), shaped like tmY.
struct Q8PeerMaps {
    CUtensorMap m[kMaxScatter];
};

__device__ __forceinline__ void put_y(const Q8Params& p, int64_t m, int64_t n, float v)
{
    p.y[m * p.ldy + n] = v;
    const int64_t off = m * p.ldy + p.col_off + n;
    for (int k = 0; k < p.ndst; k++) p.ydst[k][off] = v;
}

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }

// Tile t -> (activation tile, weight tile): groups of Q8_GROUP_M activation
// tiles, weight tiles outer within a group.
__device__ __forceinline__ void q8_tile(int64_t t, int64_t mt, int64_t nt, int64_t& mi, int64_t& ni)
{
    const int64_t per_group = (int64_t)Q8_GROUP_M * nt;
    const int64_t g = t / per_group;
    const int64_t fm = g * Q8_GROUP_M;
    const int64_t gm = mt - fm < Q8_GROUP_M ? mt - fm : Q8_GROUP_M;
    const int64_t r = t - g * per_group;
    mi = fm + r % gm;
    ni = r / gm;
}

// ---------------------------------------------------------------------------
// OPK 2: the scale products on the tensor core.  Per 32-block b, besides the
// block dots I (two kind::f16 MMAs on the exact fp16 quants), one K = 16 MMA
// of a one-hot weight-scale tile (dW[n,b] at position b % 16 of a 16-wide
// row, from the repack) against the activations' fp16 scale tile (dX[m, 16g
// .. 16g+15]) gives S[n,m] = dW[n,b] * dX[m,b] exactly (fp16 x fp16 fits
// fp32).  The drain then does one FMA per element and block, acc += S * I,
// and reads no scales from shared memory; TMEM holds (S, I) for two blocks.
// Two issuer threads (the two warps after the producer) take alternate
// blocks, one per TMEM slot pair, so one pair's wait for its release
// overlaps the other's issue; both commit to each operand stage's empty
// barrier (count 2).
constexpr int Q8S_STAGES = 3;
constexpr int Q8S_W1H = 128 * 32;                                   // one-hot tile [128][16] fp16, 32-byte swizzle
constexpr int Q8S_XS = 128 * 32;                                    // activation scale tile [128][16] fp16
// blocks per operand stage: one 128-byte swizzle row holds 2 blocks of fp16
// quants, 4 of int8 quants (operand kind 4)
template <bool I8>
__host__ __device__ constexpr int q8s_bps() { return I8 ? 4 : 2; }
// W | X | one-hot x BPS | X scales: 44 KB (fp16 quants), 52 KB (int8 quants)
template <bool I8>
__host__ __device__ constexpr int q8s_stage() { return 2 * Q8_OP_BYTES + q8s_bps<I8>() * Q8S_W1H + Q8S_XS; }
// Shared memory and TMEM of the scale-product kernels.  One-hot form (CC =
// false): 3 stages of W | X | one-hot x BPS | X scales, two TMEM slots of
// 256 columns (S, I).  CUDA-core form (CC = true): 4 stages of W | X, a ring
// of fp32 scale entries (dW | dX, [BPS][128] each) that the drain releases,
// four TMEM slots of 128 columns (I).
template <bool I8, bool CC>
struct Q8sLayout {
    static constexpr int BPS = q8s_bps<I8>();
    static constexpr int STAGE = CC ? Q8_STAGE : q8s_stage<I8>();
    static constexpr int STAGES = CC ? 4 : Q8S_STAGES;
    static constexpr int SLOTS = CC ? 4 : 2;
    static constexpr int SLOT_COLS = CC ? Q8_TM : 2 * Q8_TM;
    static constexpr int SD = CC ? Q8Op<I8 ? 1 : 0>::SD : 0;
    static constexpr int EB = CC ? q8_entry_bytes<I8 ? 1 : 0>() : 0;
    static constexpr int OFF_RING = STAGES * STAGE;
    static constexpr int OFF_STAGING = OFF_RING + SD * EB;
    static constexpr int OFF_BAR = OFF_STAGING + Q8_STAGING;
    static constexpr int NUM_BARS = 2 * STAGES + 2 * SLOTS + 2 * SD + 1 + 2;
    static constexpr int SMEM = OFF_BAR + NUM_BARS * 8 + 16 + 1024;
    static_assert(SMEM <= 232448, "shared memory");
    static_assert(STAGE % 1024 == 0, "swizzled tiles need 1024-byte alignment");
    static_assert(SLOTS * SLOT_COLS <= 512, "TMEM columns");
};

__device__ __forceinline__ uint64_t desc_sw32(uint32_t saddr) { return smem_desc(saddr, 16, 256, 6); }

// tensor maps:
//   tmW   weight operand fp16 [N][K]            box {64, 128}  128B swizzle
//   tmX   activation operand fp16 [M][K]        box {64, 128}  128B swizzle
//   tmWs  one-hot weight scales fp16 [N][nb*16] box {16, 128}  32B swizzle
//   tmXs  activation scales fp16 [M][ldd]       box {16, 128}  32B swizzle
//   tmY   output fp32 [M][ldy], box {32, 32} (TMA-store epilogue)
// Drain shapes: DW = 16 warps of 32 accumulator columns (104 registers each)
// or DW = 8 warps of 64 (232 registers), plus one warpgroup for the producer
// and the two MMA issuers.  The wider drain loads a block's S and I for its
// 64 columns at once, so per block it pays its wait / load / release once for
// twice the elements, and two warps per scheduler share the issue slots.
template <int DW>
struct Q8sDrain {
    static constexpr int WARPS = DW;
    static constexpr int GROUPS = DW / 4;                      // column groups per TMEM lane quadrant
    static constexpr int HC = Q8_TN / GROUPS;                  // accumulator columns per drain warp
    static constexpr int THREADS = (DW + 4) * 32;
    static constexpr int PRODUCER_WARP = DW, MMA_WARP = DW + 1;
    static constexpr uint32_t DRAIN_REGS = DW == 16 ? 104 : 232, PRODUCER_REGS = 40;
    // the registers a CTA launches with: 64 K per SM over THREADS, in steps of 8
    static constexpr int LAUNCH_REGS = (65536 / THREADS) / 8 * 8;
    static_assert(DW == 16 || DW == 8, "drain shape");
    static_assert(32 * DW * DRAIN_REGS + 128 * PRODUCER_REGS <= THREADS * LAUNCH_REGS, "setmaxnreg split");
    static_assert(DW * HC * 32 * 4 <= Q8_STAGING, "staging holds every drain warp's output tile");
};

template <bool DUMP, bool I8, int DW, bool CC>
__global__ void __launch_bounds__(Q8sDrain<DW>::THREADS, 1)
    k_gemm_q8s(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
               const __grid_constant__ CUtensorMap tmWs, const __grid_constant__ CUtensorMap tmXs,
               const __grid_constant__ CUtensorMap tmY, const Q8Params p, const __grid_constant__ Q8PeerMaps peers)
{
    constexpr uint32_t IDESC = idesc_f16_f32(Q8_TN, Q8_TM);
    constexpr uint32_t IDESC_I8 = idesc_i8_s32(Q8_TN, Q8_TM);
    using L = Q8sLayout<I8, CC>;
    constexpr int BPS = L::BPS, STAGE = L::STAGE, STAGES = L::STAGES, SLOTS = L::SLOTS, SD = L::SD, EB = L::EB;
    using D = Q8sDrain<DW>;
    constexpr int HC = D::HC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* full = bars;                   // operand stage loaded
    uint64_t* empty = full + STAGES;         // operand stage consumed by the MMAs
    uint64_t* tfull = empty + STAGES;        // slot holds a block's (S, I), or I alone (CC)
    uint64_t* tempty = tfull + SLOTS;        // slot read by every drain warp
    uint64_t* sfull = tempty + SLOTS;        // CC: scale entry loaded
    uint64_t* sempty = sfull + SD;           // CC: scale entry read by every drain warp
    uint64_t* mma_done = sempty + SD;
    uint64_t* merge = mma_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NUM_BARS);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    uint8_t* scale_ring = smem + L::OFF_RING;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 2);  // both MMA issuers commit
        }
        for (int i = 0; i < SLOTS; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], D::WARPS);
        }
        for (int i = 0; i < SD; i++) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sempty[i], D::WARPS);
        }
        mbar_init(mma_done, 2);
        mbar_init(&merge[0], 32 * D::WARPS);
        mbar_init(&merge[1], 32 * D::WARPS);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == D::PRODUCER_WARP && lane == 0) {
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmWs);
        tma_prefetch_desc(&tmXs);
        if (p.tma_store) tma_prefetch_desc(&tmY);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int64_t mt = (p.M + Q8_TM - 1) / Q8_TM;
    const int64_t nt = (p.N + Q8_TN - 1) / Q8_TN;
    const int64_t tiles = mt * nt;
    const int64_t nb = p.K / kQK8_0;
    const int64_t nstages = (nb + BPS - 1) / BPS;
    uint32_t* status = p.status;

    if (warp >= D::WARPS) {
        regs_dec<D::PRODUCER_REGS>();
        if (warp == D::PRODUCER_WARP && lane == 0) {
            int stage = 0, se = 0;
            uint32_t ph = 0, sph = 0;
            for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                int64_t mi, ni;
                q8_tile(tile, mt, nt, mi, ni);
                const int32_t m0 = (int32_t)(mi * Q8_TM);
                const int32_t n0 = (int32_t)(p.n_first + ni * Q8_TN);
                for (int64_t kc = 0; kc < nstages; kc++) {
                    if constexpr (CC) {
                        // the stage's block scales, for the drain: dW | dX fp32, [BPS][128] each
                        if (!mbar_wait(&sempty[se], sph ^ 1u, abort_flag, status, kDevTimeoutScaleEmpty)) goto done;
                        uint8_t* e = scale_ring + se * EB;
                        mbar_expect_tx(&sfull[se], EB);
                        tma_load_2d(e, &tmWs, &sfull[se], n0, (int32_t)(kc * BPS));
                        tma_load_2d(e + EB / 2, &tmXs, &sfull[se], m0, (int32_t)(kc * BPS));
                        if (++se == SD) {
                            se = 0;
                            sph ^= 1u;
                        }
                    }
                    if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, status, kDevTimeoutEmpty)) goto done;
                    uint8_t* st = smem + stage * STAGE;
                    const int nblk = nb - BPS * kc < BPS ? (int)(nb - BPS * kc) : BPS;
                    mbar_expect_tx(&full[stage], CC ? 2 * Q8_OP_BYTES : 2 * Q8_OP_BYTES + nblk * Q8S_W1H + Q8S_XS);
                    const int32_t kx = (int32_t)(kc * 32 * BPS);  // quants of BPS blocks: one 128-byte row
                    tma_load_2d(st, &tmW, &full[stage], kx, n0);
                    tma_load_2d(st + Q8_OP_BYTES, &tmX, &full[stage], kx, m0);
                    if constexpr (!CC) {
                        for (int b = 0; b < nblk; b++)
                            tma_load_2d(st + 2 * Q8_OP_BYTES + b * Q8S_W1H, &tmWs, &full[stage], (int32_t)((BPS * kc + b) * 16), n0);
                        tma_load_2d(st + 2 * Q8_OP_BYTES + BPS * Q8S_W1H, &tmXs, &full[stage], (int32_t)(((BPS * kc) / 16) * 16), m0);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        } else if ((warp == D::MMA_WARP || warp == D::MMA_WARP + 1) && lane == 0) {
            // two issuers take alternate blocks: block g goes to slot g % SLOTS
            // and to the issuer g % 2
            const int mine = warp - D::MMA_WARP;
            int stage = 0;
            uint32_t ph = 0;
            int64_t gb = 0;  // global block index (both issuers walk every block)
            for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                for (int64_t kc = 0; kc < nstages; kc++) {
                    if (!mbar_wait(&full[stage], ph, abort_flag, status, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(smem + stage * STAGE);
                    const uint32_t x_addr = w_addr + Q8_OP_BYTES;
                    const uint32_t ws_addr = x_addr + Q8_OP_BYTES;
                    const uint32_t xs_addr = ws_addr + BPS * Q8S_W1H;
#pragma unroll
                    for (int bi = 0; bi < BPS; bi++) {
                        if (BPS * kc + bi >= nb) break;
                        if ((int)(gb & 1) == mine) {
                            const int slot = (int)(gb % SLOTS);
                            const uint32_t tph = (uint32_t)(gb / SLOTS) & 1u;
                            if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            tc_fence_after();
                            const uint32_t ds = tmem_base + (uint32_t)(slot * L::SLOT_COLS);
                            // I: the block's dots, in the slot's last 128 columns
                            const uint32_t di = ds + (CC ? 0u : (uint32_t)Q8_TM);
                            if constexpr (!CC) {
                                if (!DUMP) mma_f16(ds, desc_sw32(ws_addr + bi * Q8S_W1H), desc_sw32(xs_addr), IDESC, 0u);
                            }
                            if constexpr (I8) {
                                const uint32_t koff = (uint32_t)bi * 32u;
                                mma_i8(di, desc_sw128(w_addr + koff), desc_sw128(x_addr + koff), IDESC_I8, 0u);
                            } else {
#pragma unroll
                                for (int k = 0; k < 2; k++) {
                                    const uint32_t koff = (uint32_t)(bi * 2 + k) * 32u;
                                    mma_f16(di, desc_sw128(w_addr + koff), desc_sw128(x_addr + koff), IDESC, (uint32_t)k);
                                }
                            }
                            mma_commit(&tfull[slot]);
                        }
                        gb++;
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
        regs_inc<D::DRAIN_REGS>();
        const uint32_t quad = warp & 3u, quarter = warp >> 2;  // lane quadrant, column group
        const uint32_t lane_base = (quad * 32u) << 16;
        const uint32_t col0 = quarter * HC;
        const uint32_t t_row = tmem_base + lane_base + col0;  // this warp's lanes and columns in slot 0
        const int nb32 = (int)nb;                             // the host caps K at INT32_MAX
        int slot = 0, se = 0;
        uint32_t tph = 0, sph = 0, mgph = 0;
        auto drain_meet = [&](int i) -> bool {
            mbar_arrive(&merge[i]);
            return mbar_wait(&merge[i], mgph, abort_flag, status, kDevTimeoutTmemFull);
        };
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            int64_t mi, ni;
            q8_tile(tile, mt, nt, mi, ni);
            const int64_t m0 = mi * Q8_TM;
            const int64_t n0 = ni * Q8_TN;       // view-local
            const int64_t nq = n0 + quad * 32u;  // the warp's first weight row
            const int64_t n = nq + lane;         // this thread's weight row == TMEM lane
            const int64_t mfirst = m0 + col0;
            float acc[HC];
#pragma unroll
            for (int i = 0; i < HC; i++) acc[i] = 0.f;
            for (int b = 0; b < nb32; b++) {
                const int bi = b % BPS;
                if (CC && bi == 0 && !mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                if (!mbar_wait(&tfull[slot], tph, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                tc_fence_after();
                const uint32_t ts = t_row + (uint32_t)(slot * L::SLOT_COLS);
                uint32_t sv[CC ? 1 : HC], iv[HC];
#pragma unroll
                for (int c = 0; c < HC; c += 32) {
                    if constexpr (!CC) {
                        if (!DUMP) tmem_ld32(ts + c, *reinterpret_cast<uint32_t(*)[32]>(sv + c));
                    }
                    tmem_ld32(ts + (CC ? 0u : (uint32_t)Q8_TM) + c, *reinterpret_cast<uint32_t(*)[32]>(iv + c));
                }
                // CC: this block's weight scale (the thread's row) and the warp's
                // activation scales, from the scale entry
                const float* se_w = reinterpret_cast<const float*>(scale_ring + se * EB) + bi * 128;
                const float* se_x = reinterpret_cast<const float*>(scale_ring + se * EB + EB / 2) + bi * 128 + col0;
                const float dwv = CC ? se_w[quad * 32u + lane] : 0.f;
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[slot]);
                if (++slot == SLOTS) {
                    slot = 0;
                    tph ^= 1u;
                }
                if constexpr (DUMP) {
#pragma unroll
                    for (int j = 0; j < HC; j++) {
                        const int64_t m = mfirst + j;
                        if (n < p.N && m < p.M)
                            p.dump[((int64_t)b * p.M + m) * p.N + n] = I8 ? __int2float_rn((int)iv[j]) : __uint_as_float(iv[j]);
                    }
                } else if constexpr (CC) {
                    // pix_dot_q8_0: S = fp16(dw)*fp16(dx) (exact in fp32), acc = fma(S, float(block dot), acc),
                    // two per instruction; the activation scales are shared-memory broadcasts
#pragma unroll
                    for (int j = 0; j < HC; j += 4) {
                        const float4 dx4 = *reinterpret_cast<const float4*>(se_x + j);
                        float s0, s1, s2, s3;
                        fmul2(s0, s1, dx4.x, dx4.y, dwv, dwv);
                        fmul2(s2, s3, dx4.z, dx4.w, dwv, dwv);
                        const float i0 = I8 ? __int2float_rn((int)iv[j]) : __uint_as_float(iv[j]);
                        const float i1 = I8 ? __int2float_rn((int)iv[j + 1]) : __uint_as_float(iv[j + 1]);
                        const float i2 = I8 ? __int2float_rn((int)iv[j + 2]) : __uint_as_float(iv[j + 2]);
                        const float i3 = I8 ? __int2float_rn((int)iv[j + 3]) : __uint_as_float(iv[j + 3]);
                        ffma2(acc[j], acc[j + 1], s0, s1, i0, i1);
                        ffma2(acc[j + 2], acc[j + 3], s2, s3, i2, i3);
                    }
                } else {
                    // pix_dot_q8_0: acc = fma(fp16(dw)*fp16(dx), float(block dot), acc), two per instruction
#pragma unroll
                    for (int j = 0; j < HC; j += 2) {
                        // kind::i8 leaves exact int32 dots: |I| <= 32 * 127 * 127, exact in fp32
                        const float i0 = I8 ? __int2float_rn((int)iv[j]) : __uint_as_float(iv[j]);
                        const float i1 = I8 ? __int2float_rn((int)iv[j + 1]) : __uint_as_float(iv[j + 1]);
                        ffma2(acc[j], acc[j + 1], __uint_as_float(sv[j]), __uint_as_float(sv[j + 1]), i0, i1);
                    }
                }
                if (CC && (bi == BPS - 1 || b + 1 == nb32)) {
                    // every lane's scale reads are done before lane 0 frees the entry
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sempty[se]);
                    if (++se == SD) {
                        se = 0;
                        sph ^= 1u;
                    }
                }
            }
            if constexpr (!DUMP) {
                if (p.gated) {
                    // gated weight: lanes 64..127 hold the up projections of the
                    // outputs whose gate projections lanes 0..63 hold (the repack
                    // interleaves 64-row groups); the up warps hand their sums over
                    // through the staging buffer and the gate warps finish
                    // tensor_silu + tensor_gate (src/tensor.cpp:199-208, :334-345)
                    float* xfer = reinterpret_cast<float*>(smem + L::OFF_STAGING) + ((quad & 1) * D::GROUPS + quarter) * (HC * 32);
                    if (!drain_meet(0)) goto done;
                    if (quad >= 2) {
#pragma unroll
                        for (int i = 0; i < HC; i++) xfer[i * 32 + lane] = acc[i];
                    }
                    if (!drain_meet(1)) goto done;
                    mgph ^= 1u;
                    if (quad < 2) {
#pragma unroll
                        for (int i = 0; i < HC; i++) {
                            const int64_t on = n0 / 2 + quad * 32 + lane, m = mfirst + i;
                            const float g = acc[i], u = xfer[i * 32 + lane];
                            if (on < p.N / 2 && m < p.M) p.y[m * p.ldy + on] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                        }
                    }
                    continue;
                }
                const float bv = (p.bias && n < p.N) ? p.bias[n] : 0.f;
                if (p.tma_store) {
                    float* stg = reinterpret_cast<float*>(smem + L::OFF_STAGING) + warp * (HC * 32);
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < HC; j++) stg[j * 32 + lane] = p.bias ? __fadd_rn(acc[j], bv) : acc[j];
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
#pragma unroll
                        for (int c = 0; c < HC; c += 32) tma_store_2d(&tmY, stg + c * 32, (int32_t)nq, (int32_t)(mfirst + c));
                        // the scatter: the same boxes into every destination, asynchronous
                        // like the local store (peers' memory over NVLink)
                        if (p.tma_dst)
                            for (int k = 0; k < p.ndst; k++)
#pragma unroll
                                for (int c = 0; c < HC; c += 32)
                                    tma_store_2d(&peers.m[k], stg + c * 32, (int32_t)nq, (int32_t)(mfirst + c));
                        bulk_commit();
                    }
                    if (p.tma_dst) {
                        // stored above
                    } else if (p.ndst && p.dst_vec4) {
                        const int jr = lane >> 3, c4 = 4 * (lane & 7);
                        const int64_t nn = nq + c4;
                        for (int j = jr; j < HC; j += 4) {
                            const int64_t m = mfirst + j;
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
                    } else if (p.ndst && n < p.N) {
                        for (int j = 0; j < HC; j++) {
                            const int64_t m = mfirst + j;
                            if (m >= p.M) break;
                            const float v = stg[j * 32 + lane];
                            const int64_t off = m * p.ldy + p.col_off + n;
                            for (int k = 0; k < p.ndst; k++) p.ydst[k][off] = v;
                        }
                    }
                } else if (n < p.N) {
#pragma unroll
                    for (int j = 0; j < HC; j++) {
                        const int64_t m = mfirst + j;
                        if (m < p.M) put_y(p, m, n, p.bias ? __fadd_rn(acc[j], bv) : acc[j]);
                    }
                }
            }
        }
    }
done:
    if (p.tma_store && warp < D::WARPS && lane == 0) bulk_wait_all();
    if (p.ndst && warp < D::WARPS) __threadfence_system();
    if ((warp == D::MMA_WARP || warp == D::MMA_WARP + 1) && lane == 0) {
        mma_commit(mma_done);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(mma_done, 0) && global_ns() - t0 < PXQ_WAIT_NS) {
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, 512);
}

// ---------------------------------------------------------------------------
// OPK 3: CTA pairs.  The pair's tile is 256 weight rows (the MMA's M; each
// CTA stages and accumulates its 128) by 256 activation rows (the MMA's N;
// each CTA stages 128 of them and receives all 256 columns in its TMEM), so
// per block an SM drains 128 x 256 block dots and streams 16 KB of fp16
// operands for them -- half the operand bytes per output of the one-CTA
// kinds.  Two 256-column accumulator slots alternate per 32-block.  The
// drain reads each block dot once from TMEM (32x32b layout: a thread holds
// one weight row, whose scale is a register, and 128 activation rows, whose
// scales are shared-memory broadcasts) and does two packed fp32 operations
// per element pair: S = dX * dW, acc = fma(S, I, acc).  That FP32 work --
// 2 * 128 * 256 lane operations per block and SM, 512 clocks at 128 lanes
// per clock -- is the kernel's floor; the MMAs (292 clocks per block on the
// f16 pipe) and the TMEM reads (about 280) fit beside it.
//   Roles (12 warps): warps 0-7 drain (warp w: TMEM lane quadrant w % 4,
//   columns 128 * (w / 4) ..+128); warp 8 loads (both CTAs); warp 9 of the
//   even CTA issues the pair MMAs.  Barriers as in gemm.cu's pair kernel:
//   both CTAs' stage loads complete on the even CTA's stage barrier, its
//   commits arrive on both CTAs' barriers, the odd CTA's drain releases slots
//   on the even CTA's barriers.
constexpr int Q8P_TN = 128;                         // weight rows per CTA (TMEM lanes)
constexpr int Q8P_TMP = 256;                        // activation rows per pair tile (TMEM columns per slot)
constexpr int Q8P_XR = 128;                         // activation rows staged per CTA
constexpr int Q8P_STAGE = 2 * Q8_OP_BYTES;          // W [128][64 fp16] | X [128][64 fp16], 128B swizzle: 32 KB
constexpr int Q8P_STAGES = 4;
constexpr int Q8P_BPS = 2;                          // 32-blocks per stage and per scale entry
constexpr int Q8P_SE = 8;                           // scale entries
constexpr int Q8P_ENTRY = Q8P_BPS * (Q8P_TN + Q8P_TMP) * 4;  // dW [2][128] | dX [2][256] fp32: 3 KB
constexpr int Q8P_DX_OFF = Q8P_BPS * Q8P_TN * 4;
constexpr int Q8P_DRAIN = 8;
constexpr int Q8P_THREADS = 32 * (Q8P_DRAIN + 4);
constexpr int Q8P_PRODUCER_WARP = Q8P_DRAIN, Q8P_MMA_WARP = Q8P_DRAIN + 1;
constexpr int Q8P_HC = Q8P_TMP / (Q8P_DRAIN / 4);    // TMEM columns per drain warp: 128
constexpr int Q8P_CW = 16;                          // columns per TMEM load
constexpr int Q8P_STG_BUFS = 2;                     // output staging buffers per drain warp
// the drain's 128 accumulators, two loads and their scales need 232 registers
constexpr uint32_t Q8P_DRAIN_REGS = 232, Q8P_PRODUCER_REGS = 40;
static_assert(256 * Q8P_DRAIN_REGS + 128 * Q8P_PRODUCER_REGS <= Q8P_THREADS * 168, "setmaxnreg split");
constexpr int Q8P_OFF_SCALES = Q8P_STAGES * Q8P_STAGE;
constexpr int Q8P_OFF_STAGING = Q8P_OFF_SCALES + Q8P_SE * Q8P_ENTRY;
constexpr int Q8P_STAGING = Q8P_DRAIN * Q8P_STG_BUFS * 32 * 32 * 4;  // [32 activation rows][32 weight rows] fp32 buffers
constexpr int Q8P_OFF_BAR = Q8P_OFF_STAGING + Q8P_STAGING;
// full/empty, scale full/empty, slot full/empty, MMA drain-out, gated hand-over
constexpr int Q8P_NUM_BARS = 2 * Q8P_STAGES + 2 * Q8P_SE + 2 * 2 + 1 + 2;
constexpr int Q8P_SMEM = Q8P_OFF_BAR + Q8P_NUM_BARS * 8 + 16 + 1024;
static_assert(Q8P_SMEM <= 232448, "shared memory");
static_assert(Q8P_STAGE % 1024 == 0 && Q8P_OFF_SCALES % 1024 == 0 && Q8P_ENTRY % 128 == 0, "alignment");
static_assert(2 * Q8P_TMP <= 512, "TMEM columns");
static_assert(Q8P_STAGING >= 2 * (Q8P_DRAIN / 4) * Q8P_HC * 32 * 4, "gated hand-over buffer");

// acc[j] += (dx[j] * dw) * I[j] over one TMEM load's columns, two per instruction
// (pix_dot_q8_0: the fp32 product of the two fp16 scales, exact, times the
// exact block dot, accumulated with one rounding).  dx: the columns' scales,
// loaded from shared memory one load ahead (q8p_dx).
__device__ __forceinline__ void q8p_dx(float4 (&d)[Q8P_CW / 4], const float* dx)
{
#pragma unroll
    for (int j = 0; j < Q8P_CW / 4; j++) d[j] = reinterpret_cast<const float4*>(dx)[j];
}
__device__ __forceinline__ void q8p_fma(float* acc, const uint32_t (&v)[Q8P_CW], const float4 (&d)[Q8P_CW / 4], float dw)
{
#pragma unroll
    for (int j = 0; j < Q8P_CW; j += 4) {
        const float4 d4 = d[j / 4];
        float s0, s1, s2, s3;
        fmul2(s0, s1, d4.x, d4.y, dw, dw);
        fmul2(s2, s3, d4.z, d4.w, dw, dw);
        ffma2(acc[j], acc[j + 1], s0, s1, __uint_as_float(v[j]), __uint_as_float(v[j + 1]));
        ffma2(acc[j + 2], acc[j + 3], s2, s3, __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
    }
}

// tensor maps:
//   tmW   weight operand fp16 [N][K]             box {64, 128}  128B swizzle
//   tmX   activation operand fp16 [M][K]         box {64, 128}  128B swizzle
//   tmDw  weight block scales fp32 [K/32][ldn]   box {128, 2}
//   tmDx  activation block scales fp32 [K/32][ldm] box {256, 2}
//   tmY   output fp32 [M][ldy], box {32, 32} (TMA-store epilogue)
template <bool DUMP>
__global__ void __launch_bounds__(Q8P_THREADS, 1)
    k_gemm_q8p(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
               const __grid_constant__ CUtensorMap tmDw, const __grid_constant__ CUtensorMap tmDx,
               const __grid_constant__ CUtensorMap tmY, const Q8Params p)
{
    constexpr uint32_t IDESC = idesc_f16_f32(2 * Q8P_TN, Q8P_TMP);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q8P_OFF_BAR);
    uint64_t* full = bars;                   // even CTA: stage loaded (both CTAs' bytes)
    uint64_t* empty = full + Q8P_STAGES;     // stage consumed by the MMAs (both CTAs)
    uint64_t* sfull = empty + Q8P_STAGES;    // this CTA's scale entry loaded
    uint64_t* sempty = sfull + Q8P_SE;       // ... and read by this CTA's drain warps
    uint64_t* tfull = sempty + Q8P_SE;       // slot holds a finished block (both CTAs)
    uint64_t* tempty = tfull + 2;            // even CTA: slot read by both CTAs' drain warps
    uint64_t* mma_done = tempty + 2;         // even CTA: every issued MMA finished (exit path)
    uint64_t* merge = mma_done + 1;          // gated epilogue hand-over
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Q8P_NUM_BARS);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    uint8_t* scale_ring = smem + Q8P_OFF_SCALES;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Q8P_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < Q8P_SE; i++) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sempty[i], Q8P_DRAIN);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 2 * Q8P_DRAIN);  // the drain warps of both CTAs
        }
        mbar_init(mma_done, 1);
        mbar_init(&merge[0], 32 * Q8P_DRAIN);
        mbar_init(&merge[1], 32 * Q8P_DRAIN);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    if (warp == Q8P_PRODUCER_WARP && lane == 0) {
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmDw);
        tma_prefetch_desc(&tmDx);
        if (p.tma_store) tma_prefetch_desc(&tmY);
    }
    // barriers initialised and TMEM allocated in both CTAs before any cross-CTA traffic
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int64_t mt = (p.M + Q8P_TMP - 1) / Q8P_TMP;
    const int64_t nt = (p.N + 2 * Q8P_TN - 1) / (2 * Q8P_TN);
    const int64_t tiles = mt * nt;
    const int64_t pair = (int64_t)cluster_id_x(), pairs = (int64_t)cluster_count_x();
    const int64_t nb = p.K / kQK8_0;
    const int64_t nstages = (nb + Q8P_BPS - 1) / Q8P_BPS;
    uint32_t* status = p.status;

    if (warp >= Q8P_DRAIN) {
        regs_dec<Q8P_PRODUCER_REGS>();
        if (warp == Q8P_PRODUCER_WARP && lane == 0) {
            const uint32_t full0 = cluster_map(smem_u32(full), 0);  // the even CTA's stage barriers
            int stage = 0, se = 0;
            uint32_t ph = 0, sph = 0;
            for (int64_t tile = pair; tile < tiles; tile += pairs) {
                int64_t mi, ni;
                q8_tile(tile, mt, nt, mi, ni);
                const int32_t m0 = (int32_t)(mi * Q8P_TMP);
                const int32_t mc = m0 + (int32_t)(rank * Q8P_XR);
                const int32_t nc = (int32_t)(p.n_first + ni * 2 * Q8P_TN + rank * Q8P_TN);
                for (int64_t kc = 0; kc < nstages; kc++) {
                    // this CTA's block scales for its drain: its 128 weight rows, all 256 activation rows
                    if (!mbar_wait(&sempty[se], sph ^ 1u, abort_flag, status, kDevTimeoutScaleEmpty)) goto done;
                    uint8_t* e = scale_ring + se * Q8P_ENTRY;
                    mbar_expect_tx(&sfull[se], Q8P_ENTRY);
                    tma_load_2d(e, &tmDw, &sfull[se], nc, (int32_t)(kc * Q8P_BPS));
                    tma_load_2d(e + Q8P_DX_OFF, &tmDx, &sfull[se], m0, (int32_t)(kc * Q8P_BPS));
                    if (++se == Q8P_SE) {
                        se = 0;
                        sph ^= 1u;
                    }
                    // this CTA's halves of the stage's operands, reported to the even CTA
                    if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, status, kDevTimeoutEmpty)) goto done;
                    uint8_t* st = smem + stage * Q8P_STAGE;
                    if (leader) mbar_expect_tx(&full[stage], 2 * Q8P_STAGE);
                    const int32_t kx = (int32_t)(kc * 64);
                    tma_load_2d_pair(st, &tmW, full0 + 8u * stage, kx, nc);
                    tma_load_2d_pair(st + Q8_OP_BYTES, &tmX, full0 + 8u * stage, kx, mc);
                    if (++stage == Q8P_STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        } else if (warp == Q8P_MMA_WARP && lane == 0 && leader) {
            int stage = 0, slot = 0;
            uint32_t ph = 0, tph = 0;
            for (int64_t tile = pair; tile < tiles; tile += pairs) {
                for (int64_t kc = 0; kc < nstages; kc++) {
                    if (!mbar_wait(&full[stage], ph, abort_flag, status, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(smem + stage * Q8P_STAGE);
                    const uint32_t x_addr = w_addr + Q8_OP_BYTES;
#pragma unroll
                    for (int bi = 0; bi < Q8P_BPS; bi++) {
                        if (kc * Q8P_BPS + bi >= nb) break;
                        if (!mbar_wait_cluster(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                        tc_fence_after();
                        const uint32_t d = tmem_base + (uint32_t)(slot * Q8P_TMP);
#pragma unroll
                        for (int k = 0; k < 2; k++) {
                            const uint32_t koff = (uint32_t)(bi * 2 + k) * 32u;  // 16 fp16 of K per MMA
                            mma_f16_pair(d, desc_sw128(w_addr + koff), desc_sw128(x_addr + koff), IDESC, (uint32_t)k);
                        }
                        mma_commit_pair(&tfull[slot]);
                        if (++slot == 2) {
                            slot = 0;
                            tph ^= 1u;
                        }
                    }
                    mma_commit_pair(&empty[stage]);
                    if (++stage == Q8P_STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------ drain warps --
        regs_inc<Q8P_DRAIN_REGS>();
        const uint32_t quad = warp & 3u, half = warp >> 2;  // half: the warp's column group
        const uint32_t lane_base = (quad * 32u) << 16;
        const uint32_t tempty0 = cluster_map(smem_u32(tempty), 0);  // the even CTA's slot barriers
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
        int slot = 0, se = 0;
        uint32_t tph = 0, sph = 0, mgph = 0;
        auto drain_meet = [&](int i) -> bool {
            mbar_arrive(&merge[i]);
            return mbar_wait(&merge[i], mgph, abort_flag, status, kDevTimeoutTmemFull);
        };
        constexpr int NCH = Q8P_HC / Q8P_CW;
        for (int64_t tile = pair; tile < tiles; tile += pairs) {
            int64_t mi, ni;
            q8_tile(tile, mt, nt, mi, ni);
            const int64_t m0 = mi * Q8P_TMP;
            const int64_t n0 = ni * 2 * Q8P_TN + rank * Q8P_TN;  // view-local, this CTA's first weight row
            const int64_t nq = n0 + quad * 32u;                   // the warp's first weight row
            const int64_t n = nq + lane;                          // this thread's weight row == TMEM lane
            const int64_t mfirst = m0 + half * Q8P_HC;
            float acc[Q8P_HC];
#pragma unroll
            for (int i = 0; i < Q8P_HC; i++) acc[i] = 0.f;
            for (int64_t b = 0; b < nb; b++) {
                const int bi = (int)(b % Q8P_BPS);
                if (bi == 0 && !mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                const float* ef = reinterpret_cast<const float*>(scale_ring + se * Q8P_ENTRY);
                const float dw = ef[bi * Q8P_TN + quad * 32u + lane];
                const float* dx = ef + Q8P_BPS * Q8P_TN + bi * Q8P_TMP + half * Q8P_HC;
                if (!mbar_wait(&tfull[slot], tph, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                tc_fence_after();
                const uint32_t taddr = tmem_base + lane_base + (uint32_t)(slot * Q8P_TMP) + half * Q8P_HC;
                if constexpr (DUMP) {
#pragma unroll 1
                    for (int c = 0; c < NCH; c++) {
                        uint32_t v[Q8P_CW];
                        tmem_ld16(taddr + (uint32_t)(c * Q8P_CW), v);
                        tmem_ld_wait_dep(v);
#pragma unroll
                        for (int j = 0; j < Q8P_CW; j++) {
                            const int64_t m = mfirst + c * Q8P_CW + j;
                            if (n < p.N && m < p.M) p.dump[(b * p.M + m) * p.N + n] = __uint_as_float(v[j]);
                        }
                    }
                    release(slot);
                } else {
                    // chunk c+1 loads while chunk c is accumulated; the slot is
                    // released once its last chunk is in registers
                    // chunk c+1 (its block dots from TMEM, its scales from shared
                    // memory) loads while chunk c is accumulated
                    uint32_t va[Q8P_CW], vb[Q8P_CW];
                    float4 xa[Q8P_CW / 4], xb[Q8P_CW / 4];
                    tmem_ld16(taddr, va);
                    q8p_dx(xa, dx);
                    tmem_ld_wait_dep(va);
#pragma unroll
                    for (int c = 0; c < NCH; c += 2) {
                        tmem_ld16(taddr + (uint32_t)((c + 1) * Q8P_CW), vb);
                        q8p_dx(xb, dx + (c + 1) * Q8P_CW);
                        q8p_fma(acc + c * Q8P_CW, va, xa, dw);
                        tmem_ld_wait_dep(vb);
                        if (c + 2 < NCH) {
                            tmem_ld16(taddr + (uint32_t)((c + 2) * Q8P_CW), va);
                            q8p_dx(xa, dx + (c + 2) * Q8P_CW);
                        } else {
                            release(slot);
                        }
                        q8p_fma(acc + (c + 1) * Q8P_CW, vb, xb, dw);
                        if (c + 2 < NCH) tmem_ld_wait_dep(va);
                    }
                }
                if (++slot == 2) {
                    slot = 0;
                    tph ^= 1u;
                }
                if (bi == Q8P_BPS - 1 || b + 1 == nb) {
                    // every lane's scale reads are done before lane 0 frees the entry
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sempty[se]);
                    if (++se == Q8P_SE) {
                        se = 0;
                        sph ^= 1u;
                    }
                }
            }
            if constexpr (!DUMP) {
                if (p.gated) {
                    // gated weight: this CTA's lanes 64..127 hold the up projections of
                    // the outputs whose gate projections lanes 0..63 hold (the repack
                    // interleaves 64-row groups); the up warps hand their sums over
                    // through the staging buffer and the gate warps finish
                    // tensor_silu + tensor_gate (src/tensor.cpp:199-208, :334-345)
                    float* xfer = reinterpret_cast<float*>(smem + Q8P_OFF_STAGING) + ((quad & 1) * (Q8P_DRAIN / 4) + half) * (Q8P_HC * 32);
                    if (!drain_meet(0)) goto done;
                    if (quad >= 2) {
#pragma unroll
                        for (int i = 0; i < Q8P_HC; i++) xfer[i * 32 + lane] = acc[i];
                    }
                    if (!drain_meet(1)) goto done;
                    mgph ^= 1u;
                    if (quad < 2) {
                        const int64_t on = n0 / 2 + quad * 32 + lane;
#pragma unroll
                        for (int i = 0; i < Q8P_HC; i++) {
                            const int64_t m = mfirst + i;
                            const float g = acc[i], u = xfer[i * 32 + lane];
                            if (on < p.N / 2 && m < p.M) p.y[m * p.ldy + on] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                        }
                    }
                    continue;
                }
                const float bv = (p.bias && n < p.N) ? p.bias[n] : 0.f;
                if (p.tma_store) {
                    // four rounds of [32 activation rows][32 weight rows], double-buffered
                    // per warp: lane 0 waits only for the store two rounds back
                    float* stg0 = reinterpret_cast<float*>(smem + Q8P_OFF_STAGING) + warp * (Q8P_STG_BUFS * 32 * 32);
#pragma unroll
                    for (int r = 0; r < Q8P_HC / 32; r++) {
                        float* stg = stg0 + (r % Q8P_STG_BUFS) * (32 * 32);
                        const int64_t mr = mfirst + 32 * r;
                        if (lane == 0) bulk_wait_read_1();
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 32; j++) stg[j * 32 + lane] = p.bias ? __fadd_rn(acc[32 * r + j], bv) : acc[32 * r + j];
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmY, stg, (int32_t)nq, (int32_t)mr);
                            bulk_commit();
                        }
                        if (p.ndst && p.dst_vec4) {
                            // the peers' copies from the same staged block, 4 floats a lane
                            const int jr = lane >> 3, c4 = 4 * (lane & 7);
                            const int64_t nn = nq + c4;
                            for (int j = jr; j < 32; j += 4) {
                                const int64_t m = mr + j;
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
                        } else if (p.ndst && n < p.N) {
                            for (int j = 0; j < 32; j++) {
                                const int64_t m = mr + j;
                                if (m >= p.M) break;
                                const float v = stg[j * 32 + lane];
                                const int64_t off = m * p.ldy + p.col_off + n;
                                for (int k = 0; k < p.ndst; k++) p.ydst[k][off] = v;
                            }
                        }
                    }
                } else if (n < p.N) {
#pragma unroll
                    for (int j = 0; j < Q8P_HC; j++) {
                        const int64_t m = mfirst + j;
                        if (m < p.M) put_y(p, m, n, p.bias ? __fadd_rn(acc[j], bv) : acc[j]);
                    }
                }
            }
        }
    }
done:
    // outstanding output stores must finish reading shared memory before exit
    if (p.tma_store && warp < Q8P_DRAIN && lane == 0) bulk_wait_all();
    // peer stores are visible system-wide before the kernel ends
    if (p.ndst && warp < Q8P_DRAIN) __threadfence_system();
    if (warp == Q8P_MMA_WARP && lane == 0 && leader) {
        // no MMA of this pair may still be writing TMEM when it is freed (after a
        // normal run the drains have consumed every result; this covers aborts)
        mma_commit_pair_local(mma_done);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(mma_done, 0) && global_ns() - t0 < PXQ_WAIT_NS) {
        }
    }
    __syncwarp();
    // the peer CTA no longer touches this CTA's barriers or TMEM after this
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp == 0) tmem_dealloc_pair(tmem_base, 512);
}

template <bool DUMP>
cudaError_t launch_q8p(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    auto kern = k_gemm_q8p<DUMP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8P_SMEM);
    if (e != cudaSuccess) return e;
    const int64_t tiles = ((op.M + Q8P_TMP - 1) / Q8P_TMP) * ((op.N + 2 * Q8P_TN - 1) / (2 * Q8P_TN));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(Q8P_THREADS);
    cfg.dynamicSmemBytes = Q8P_SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
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
    int64_t groups = max_pairs;
    if (tiles < groups) groups = tiles;
    if (groups < 1) groups = 1;
    cfg.gridDim = dim3((unsigned)(2 * groups));
    Q8Params p{op.M, op.N, op.K, op.n_first, op.y, op.ldy, op.bias, op.dump, op.status, (op.tma_store && !DUMP) ? 1 : 0,
               op.gated, op.ndst, op.dst_vec4, op.col_off, {}};
    for (int k = 0; k < kMaxScatter; k++) p.ydst[k] = op.ydst[k];
    return cudaLaunchKernelEx(&cfg, kern, op.tm[0], op.tm[1], op.tm[4], op.tm[6], op.tm_y, p);
}

template <bool DUMP, bool I8, int DW, bool CC>
cudaError_t launch_q8s(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    auto kern = k_gemm_q8s<DUMP, I8, DW, CC>;
    constexpr int smem = Q8sLayout<I8, CC>::SMEM;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int64_t tiles = ((op.M + Q8_TM - 1) / Q8_TM) * ((op.N + Q8_TN - 1) / Q8_TN);
    int64_t grid = num_sms;
    if (tiles < grid) grid = tiles;
    if (grid < 1) grid = 1;
    Q8Params p{op.M, op.N, op.K, op.n_first, op.y, op.ldy, op.bias, op.dump, op.status, (op.tma_store && !DUMP) ? 1 : 0,
               op.gated, op.ndst, op.dst_vec4, op.col_off, {}, (op.tma_dst && op.tma_store && !DUMP) ? 1 : 0};
    for (int k = 0; k < kMaxScatter; k++) p.ydst[k] = op.ydst[k];
    Q8PeerMaps peers;
    for (int k = 0; k < kMaxScatter; k++) peers.m[k] = op.tm_ydst[k];
    // tensor maps: W, X, then the one-hot and activation-scale tiles (CC =
    // false) or the fp32 block-scale planes (CC = true)
    if constexpr (CC)
        kern<<<(unsigned)grid, Q8sDrain<DW>::THREADS, smem, s>>>(op.tm[0], op.tm[1], op.tm[4], op.tm[6], op.tm_y, p, peers);
    else
        kern<<<(unsigned)grid, Q8sDrain<DW>::THREADS, smem, s>>>(op.tm[0], op.tm[1], op.tm[2], op.tm[3], op.tm_y, p, peers);
    return cudaGetLastError();
}

// Drain width of the scale-product kernels: eight 64-column drain warps (the
// faster measured), or sixteen 32-column ones with PXQ_Q8_0_DRAIN=16.
int q8s_drain_warps()
{
    static const int dw = [] {
        const char* e = getenv("PXQ_Q8_0_DRAIN");
        return (e && strcmp(e, "16") == 0) ? 16 : 8;
    }();
    return dw;
}

template <bool I8>
cudaError_t launch_q8s_any(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    if (q8s_drain_warps() == 8)
        return op.dump ? launch_q8s<true, I8, 8, false>(op, num_sms, s) : launch_q8s<false, I8, 8, false>(op, num_sms, s);
    return op.dump ? launch_q8s<true, I8, 16, false>(op, num_sms, s) : launch_q8s<false, I8, 16, false>(op, num_sms, s);
}


}  // namespace

cudaError_t launch_gemm_q8(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    if (op.q8_kind == 3) return op.dump ? launch_q8p<true>(op, num_sms, s) : launch_q8p<false>(op, num_sms, s);
    if (op.q8_kind == 2) return launch_q8s_any<false>(op, num_sms, s);
    if (op.q8_kind == 4) return launch_q8s_any<true>(op, num_sms, s);
    if (op.q8_kind == 1)
        return op.dump ? launch_q8s<true, true, 8, true>(op, num_sms, s) : launch_q8s<false, true, 8, true>(op, num_sms, s);
    return op.dump ? launch_q8s<true, false, 8, true>(op, num_sms, s) : launch_q8s<false, false, 8, true>(op, num_sms, s);
}

int gemm_q8_scale_box(int kind) { return kind == 1 ? Q8Op<1>::BPS : Q8Op<0>::BPS; }

}  // namespace pxq
