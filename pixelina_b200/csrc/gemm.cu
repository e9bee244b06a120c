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
//     64-value chunk), and its fp32 result feeds the scale FMA with no
//     int->float conversion.  (kind::i8 would double MMA throughput but its
//     int32 results need a conversion per element per block on the CUDA
//     cores, which are the bottleneck here.)
//   * Q5_K's 6-bit sub-block scales are folded into the weight operand
//     (sc*q5 <= 1953 is exact in fp16), so one MMA item covers 64 K-values;
//     the min term sum_j m_j*bsum_j is a separate K=16 MMA per super-block on
//     exact (hi, lo) splits of the activation sums.
//   * Warp roles: warps 0-7 drain TMEM and apply scales (warp w reads TMEM
//     lane quadrant w%4, column half w/4), warp 8 issues TMA loads, warp 9
//     issues MMAs.  Persistent CTAs walk 128x256 output tiles.
//   * Pipelines: 4-stage operand ring (TMA -> MMA), scale ring (TMA ->
//     drain, and -> MMA for the Q5_K min operands), two 256-column TMEM
//     slots (MMA -> drain).  All waits are time-bounded (pxq_device.cuh).
//   * Every CTA loads its own tiles from this GPU's HBM; no cluster
//     broadcast of any kind is used, so the kernel is safe in multi-GPU jobs.
#include <cuda.h>
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;              // fp16 elements per stage row (128 bytes)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int DRAIN_WARPS = 8;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int THREADS = 320;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_f16_f32(BM, BN);

// scale ring entries
constexpr int Q80_SX = BM * 2 * 4;     // dX for 2 blocks
constexpr int Q80_SW = BN * 2 * 4;     // dW for 2 blocks
constexpr int Q80_ENTRY = Q80_SX + Q80_SW;
constexpr int Q80_SDEPTH = 4;
constexpr int Q5_AMIN = BM * 32;       // [128][16] fp16, 32-byte swizzle
constexpr int Q5_BMIN = BN * 32;       // [256][16] fp16
constexpr int Q5_SX = BM * 4;
constexpr int Q5_SW = BN * 4;
constexpr int Q5_ENTRY = Q5_AMIN + Q5_BMIN + Q5_SX + 2 * Q5_SW;  // 14848
constexpr int Q5_SDEPTH = 2;
constexpr int SCALE_REGION = Q5_ENTRY * Q5_SDEPTH;  // >= Q80_ENTRY * Q80_SDEPTH
static_assert(SCALE_REGION >= Q80_ENTRY * Q80_SDEPTH, "scale region");

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
constexpr int OFF_S = OFF_B + STAGES * B_BYTES;
constexpr int OFF_BAR = OFF_S + SCALE_REGION;
constexpr int NUM_BARS = 4 * STAGES + 4;  // full/empty, sfull/sempty (<=4), tfull/tempty (2)
constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;  // + tmem addr, abort flag, alignment slack

struct Params {
    int64_t M, N, K;
    int64_t n_first;
    float* y;
    int64_t ldy;
    const float* bias;
    float* dump;
    uint32_t* status;
};

template <uint32_t TYPE>
struct Cfg;
template <>
struct Cfg<kTypeQ8_0> {
    static constexpr int SDEPTH = Q80_SDEPTH;
    static constexpr int ENTRY = Q80_ENTRY;
    static constexpr uint32_t SEMPTY_COUNT = DRAIN_WARPS;
};
template <>
struct Cfg<kTypeQ5_K> {
    static constexpr int SDEPTH = Q5_SDEPTH;
    static constexpr int ENTRY = Q5_ENTRY;
    static constexpr uint32_t SEMPTY_COUNT = DRAIN_WARPS + 1;  // drain + MMA (min operands)
};

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }
__device__ __forceinline__ uint64_t desc_sw32(uint32_t saddr) { return smem_desc(saddr, 16, 256, 6); }

template <uint32_t TYPE, bool DUMP>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
           const __grid_constant__ CUtensorMap tmSB2, const __grid_constant__ CUtensorMap tmAmin,
           const __grid_constant__ CUtensorMap tmBmin, const Params p)
{
    using C = Cfg<TYPE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* sfull = bars + 2 * STAGES;
    uint64_t* sempty = bars + 3 * STAGES;
    uint64_t* tfull = bars + 4 * STAGES;
    uint64_t* tempty = bars + 4 * STAGES + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < C::SDEPTH; i++) {
            mbar_init(&sfull[i], 1);
            mbar_init(&sempty[i], C::SEMPTY_COUNT);
        }
        for (int i = 0; i < 2; i++) {
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
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmSA);
        tma_prefetch_desc(&tmSB);
        if (TYPE == kTypeQ5_K) {
            tma_prefetch_desc(&tmSB2);
            tma_prefetch_desc(&tmAmin);
            tma_prefetch_desc(&tmBmin);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int64_t mt_count = (p.M + BM - 1) / BM;
    const int64_t nt_count = (p.N + BN - 1) / BN;
    const int64_t tiles = mt_count * nt_count;
    const int64_t nb = (TYPE == kTypeQ8_0) ? p.K / kQK8_0 : p.K / kQKK;  // blocks or super-blocks
    const int64_t nchunks = (p.K + BK - 1) / BK;
    uint32_t* status = p.status;

    if (warp == PRODUCER_WARP) {
        if (lane == 0) {
            int stage = 0;
            uint32_t ph = 0;
            int se = 0;
            uint32_t sph = 0;
            for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                const int32_t m0 = (int32_t)((tile % mt_count) * BM);
                const int32_t n0 = (int32_t)(p.n_first + (tile / mt_count) * BN);
                for (int64_t kc = 0; kc < nchunks; kc++) {
                    if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, status, kDevTimeoutEmpty)) goto done;
                    mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
                    tma_load_2d(smem + OFF_A + stage * A_BYTES, &tmA, &full[stage], (int32_t)(kc * BK), m0);
                    tma_load_2d(smem + OFF_B + stage * B_BYTES, &tmB, &full[stage], (int32_t)(kc * BK), n0);
                    const bool need_scales = (TYPE == kTypeQ8_0) || (kc % 4 == 0);
                    if (need_scales) {
                        if (!mbar_wait(&sempty[se], sph ^ 1u, abort_flag, status, kDevTimeoutScaleEmpty)) goto done;
                        uint8_t* e = smem + OFF_S + se * C::ENTRY;
                        if (TYPE == kTypeQ8_0) {
                            mbar_expect_tx(&sfull[se], Q80_ENTRY);
                            tma_load_2d(e, &tmSA, &sfull[se], m0, (int32_t)(2 * kc));
                            tma_load_2d(e + Q80_SX, &tmSB, &sfull[se], n0, (int32_t)(2 * kc));
                        } else {
                            const int32_t sb = (int32_t)(kc / 4);
                            mbar_expect_tx(&sfull[se], Q5_ENTRY);
                            tma_load_2d(e, &tmAmin, &sfull[se], sb * 16, m0);
                            tma_load_2d(e + Q5_AMIN, &tmBmin, &sfull[se], sb * 16, n0);
                            tma_load_2d(e + Q5_AMIN + Q5_BMIN, &tmSA, &sfull[se], m0, sb);
                            tma_load_2d(e + Q5_AMIN + Q5_BMIN + Q5_SX, &tmSB, &sfull[se], n0, sb);
                            tma_load_2d(e + Q5_AMIN + Q5_BMIN + Q5_SX + Q5_SW, &tmSB2, &sfull[se], n0, sb);
                        }
                        if (++se == C::SDEPTH) {
                            se = 0;
                            sph ^= 1u;
                        }
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
    } else if (warp == MMA_WARP) {
        if (lane == 0) {
            int stage = 0;
            uint32_t ph = 0;
            int slot = 0;
            uint32_t tph = 0;
            int se = 0;
            uint32_t sph = 0;
            for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
                for (int64_t kc = 0; kc < nchunks; kc++) {
                    if (!mbar_wait(&full[stage], ph, abort_flag, status, kDevTimeoutFull)) goto done;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + OFF_A + stage * A_BYTES);
                    const uint32_t b_addr = smem_u32(smem + OFF_B + stage * B_BYTES);
                    if (TYPE == kTypeQ8_0) {
#pragma unroll
                        for (int blk = 0; blk < 2; blk++) {
                            if (2 * kc + blk >= nb) break;
                            if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            tc_fence_after();
                            const uint32_t d = tmem_base + (uint32_t)slot * BN;
#pragma unroll
                            for (int k = 0; k < 2; k++) {
                                const uint32_t koff = (uint32_t)(blk * 2 + k) * 32u;  // 16 fp16 = 32 bytes
                                mma_f16(d, desc_sw128(a_addr + koff), desc_sw128(b_addr + koff), IDESC, (uint32_t)k);
                            }
                            mma_commit(&tfull[slot]);
                            if (++slot == 2) {
                                slot = 0;
                                tph ^= 1u;
                            }
                        }
                    } else {
                        if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                        tc_fence_after();
                        const uint32_t d = tmem_base + (uint32_t)slot * BN;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const uint32_t koff = (uint32_t)k * 32u;
                            mma_f16(d, desc_sw128(a_addr + koff), desc_sw128(b_addr + koff), IDESC, (uint32_t)k);
                        }
                        mma_commit(&tfull[slot]);
                        if (++slot == 2) {
                            slot = 0;
                            tph ^= 1u;
                        }
                        if (kc % 4 == 3) {
                            // min-term item of this super-block
                            if (!mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                            if (!mbar_wait(&tempty[slot], tph ^ 1u, abort_flag, status, kDevTimeoutTmemEmpty)) goto done;
                            tc_fence_after();
                            const uint32_t e = smem_u32(smem + OFF_S + se * C::ENTRY);
                            const uint32_t dm = tmem_base + (uint32_t)slot * BN;
                            mma_f16(dm, desc_sw32(e), desc_sw32(e + Q5_AMIN), IDESC, 0u);
                            mma_commit(&tfull[slot]);
                            mma_commit(&sempty[se]);
                            if (++slot == 2) {
                                slot = 0;
                                tph ^= 1u;
                            }
                            if (++se == C::SDEPTH) {
                                se = 0;
                                sph ^= 1u;
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
        const uint32_t quad = warp & 3u, half = warp >> 2;
        const uint32_t row = quad * 32u + lane;  // tile-local activation row == TMEM lane
        int slot = 0;
        uint32_t tph = 0;
        int se = 0;
        uint32_t sph = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int64_t m0 = (tile % mt_count) * BM;
            const int64_t n0 = (tile / mt_count) * BN;  // view-local
            float acc[128];
#pragma unroll
            for (int i = 0; i < 128; i++) acc[i] = 0.f;
            const int64_t n_entries = (TYPE == kTypeQ8_0) ? nchunks : nb;
            for (int64_t ent = 0; ent < n_entries; ent++) {
                if (!mbar_wait(&sfull[se], sph, abort_flag, status, kDevTimeoutScaleFull)) goto done;
                const uint8_t* e = smem + OFF_S + se * C::ENTRY;
                const int items = (TYPE == kTypeQ8_0) ? ((2 * ent + 1 < nb) ? 2 : 1) : 5;
                for (int it = 0; it < items; it++) {
                    if (!mbar_wait(&tfull[slot], tph, abort_flag, status, kDevTimeoutTmemFull)) goto done;
                    tc_fence_after();
                    float dx;
                    const float* sw;
                    if (TYPE == kTypeQ8_0) {
                        dx = reinterpret_cast<const float*>(e)[it * BM + row];
                        sw = reinterpret_cast<const float*>(e + Q80_SX) + it * BN + half * 128;
                    } else {
                        dx = reinterpret_cast<const float*>(e + Q5_AMIN + Q5_BMIN)[row];
                        sw = reinterpret_cast<const float*>(e + Q5_AMIN + Q5_BMIN + Q5_SX + (it == 4 ? Q5_SW : 0)) + half * 128;
                        if (it == 4) dx = -dx;  // min term: dmin = -y.d * fp16(x.dmin)
                    }
                    const uint32_t taddr = tmem_base + ((quad * 32u) << 16) + (uint32_t)slot * BN + half * 128u;
#pragma unroll
                    for (int c0 = 0; c0 < 128; c0 += 16) {
                        uint32_t v[16];
                        tmem_ld16(taddr + (uint32_t)c0, v);
                        tmem_ld_wait();
                        if (DUMP) {
                            const int64_t item = (TYPE == kTypeQ8_0) ? (2 * ent + it) : (ent * 5 + it);
                            const int64_t m = m0 + row;
                            if (m < p.M) {
#pragma unroll
                                for (int j = 0; j < 16; j++) {
                                    const int64_t n = n0 + half * 128 + c0 + j;
                                    if (n < p.N) p.dump[(item * p.M + m) * p.N + n] = __uint_as_float(v[j]);
                                }
                            }
                        } else {
                            const float4* s4 = reinterpret_cast<const float4*>(sw + c0);
#pragma unroll
                            for (int j4 = 0; j4 < 4; j4++) {
                                const float4 s = s4[j4];
                                acc[c0 + 4 * j4 + 0] = __fmaf_rn(__fmul_rn(dx, s.x), __uint_as_float(v[4 * j4 + 0]), acc[c0 + 4 * j4 + 0]);
                                acc[c0 + 4 * j4 + 1] = __fmaf_rn(__fmul_rn(dx, s.y), __uint_as_float(v[4 * j4 + 1]), acc[c0 + 4 * j4 + 1]);
                                acc[c0 + 4 * j4 + 2] = __fmaf_rn(__fmul_rn(dx, s.z), __uint_as_float(v[4 * j4 + 2]), acc[c0 + 4 * j4 + 2]);
                                acc[c0 + 4 * j4 + 3] = __fmaf_rn(__fmul_rn(dx, s.w), __uint_as_float(v[4 * j4 + 3]), acc[c0 + 4 * j4 + 3]);
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[slot]);
                    if (++slot == 2) {
                        slot = 0;
                        tph ^= 1u;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sempty[se]);
                if (++se == C::SDEPTH) {
                    se = 0;
                    sph ^= 1u;
                }
            }
            if (!DUMP) {
                const int64_t m = m0 + row;
                const int64_t nbase = n0 + half * 128;
                if (m < p.M) {
                    float* yr = p.y + m * p.ldy + nbase;
                    const bool fast = (nbase + 128 <= p.N) && ((p.ldy & 3) == 0) && p.bias == nullptr &&
                                      ((reinterpret_cast<uintptr_t>(p.y) & 15u) == 0);
                    if (fast) {
#pragma unroll
                        for (int c = 0; c < 128; c += 4)
                            *reinterpret_cast<float4*>(yr + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
                    } else {
#pragma unroll
                        for (int c = 0; c < 128; c++) {
                            if (nbase + c < p.N) yr[c] = p.bias ? __fadd_rn(acc[c], p.bias[nbase + c]) : acc[c];
                        }
                    }
                }
            }
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, TMEM_COLS);
}

template <uint32_t TYPE, bool DUMP>
cudaError_t launch_typed(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    auto kern = k_gemm<TYPE, DUMP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const int64_t tiles = ((op.M + BM - 1) / BM) * ((op.N + BN - 1) / BN);
    int grid = (int)(tiles < num_sms ? tiles : num_sms);
    if (grid < 1) grid = 1;
    Params p{op.M, op.N, op.K, op.n_first, op.y, op.ldy, op.bias, op.dump, op.status};
    kern<<<grid, THREADS, SMEM_BYTES, s>>>(op.tm[0], op.tm[1], op.tm[2], op.tm[3], op.tm[4], op.tm[5], op.tm[6], p);
    return cudaGetLastError();
}

}  // namespace

int gemm_smem_bytes() { return SMEM_BYTES; }

cudaError_t launch_gemm(const GemmOperands& op, int num_sms, cudaStream_t s)
{
    if (op.type == kTypeQ8_0) {
        return op.dump ? launch_typed<kTypeQ8_0, true>(op, num_sms, s) : launch_typed<kTypeQ8_0, false>(op, num_sms, s);
    }
    if (op.type == kTypeQ5_K) {
        return op.dump ? launch_typed<kTypeQ5_K, true>(op, num_sms, s) : launch_typed<kTypeQ5_K, false>(op, num_sms, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace pxq
