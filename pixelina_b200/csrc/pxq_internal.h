// pxq_internal.h -- declarations shared by the pxq translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace pxq {

constexpr int kQK8_0 = 32;        // Q8_0 block length
constexpr int kQKK = 256;         // K-quant super-block length
constexpr int kQ8_0Bytes = 34;    // {fp16 d; int8 qs[32]}
constexpr int kQ8KBytes = 292;    // {f32 d; int8 qs[256]; int16 bsums[16]}
constexpr int kQ5KBytes = 176;    // {fp16 d, dmin; u8 scales[12]; u8 qh[32]; u8 qs[128]}
constexpr int kQ6KBytes = 210;    // {u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d}
constexpr uint32_t kTypeQ8_0 = 8;
constexpr uint32_t kTypeQ5_K = 13;
constexpr uint32_t kTypeQ6_K = 14;

// ---- quantize.cu -----------------------------------------------------------
// GGUF-format activation blocks (bit-exact with the reference quantizers).
cudaError_t launch_quantize_q8_0_blocks(const float* x, void* y, int64_t rows, int64_t inner, int64_t ldx, cudaStream_t s);
cudaError_t launch_quantize_q8_K_blocks(const float* x, void* y, int64_t rows, int64_t inner, int64_t ldx, cudaStream_t s);
// Tensor-core operand formats for the GEMM (same rounding, different layout):
//   xq  fp16 [rows][inner]: the int8 quants as exact fp16 values
//   Q8_0: dx16 fp16 [rows][ldd]: the stored fp16 block scales, row-major
//   Q8_K: dxT fp32 [inner/256][ldd]: per-block scale, block-major
//         amin fp16 [rows][inner/256*16]: split 32-element sums for the Q5_K
//         min term, (hi_j, lo_j) with bsum2_j = 64*hi_j + lo_j
cudaError_t launch_quantize_q8_0_operand(const float* x, __half* xq, __half* dx16, int64_t rows, int64_t inner, int64_t ldx,
                                         int64_t ldd, cudaStream_t s);
cudaError_t launch_quantize_q8_K_operand(const float* x, __half* xq, float* dxT, __half* amin, int64_t rows, int64_t inner,
                                         int64_t ldx, int64_t ldd, cudaStream_t s);

// ---- repack.cu -------------------------------------------------------------
// One-time weight repack into the GEMM operand layout (bit-exact unpack).
cudaError_t launch_repack_q8_0(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, __half* wq, __half* ws1h,
                               cudaStream_t s);
cudaError_t launch_repack_q5_K(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, __half* wv, float* dT,
                               float* dminT, __half* bmin, int64_t ldn, cudaStream_t s);

cudaError_t launch_decode(const uint8_t* data, uint32_t type, int64_t count, float* out, cudaStream_t s);

// ---- matvec.cu -------------------------------------------------------------
// y[c*ldy + r] = dot(W row r, X row c) for c < columns <= 8, raw GGUF weights.
// The plan splits K over `ks` CTAs per 16-row group when rows are few; then
// the launch needs `partial_bytes` of fp32 workspace and `counter_bytes` of
// counters that are zero at launch (the kernel leaves them zero again).
struct MatvecPlan {
    int ks = 1;               // K slices per row group
    int chunk = 0;            // K blocks per slice
    int64_t rowgroups = 0;    // 16-row groups
    size_t smem_bytes = 0;    // dynamic shared memory per CTA
    size_t partial_bytes = 0; // split-K workspace (0 when ks == 1)
    size_t counter_bytes = 0;
};
MatvecPlan plan_matvec(uint32_t type, int64_t rows, int64_t inner, int64_t columns, int num_sms);
cudaError_t launch_matvec(uint32_t type, const uint8_t* w, int64_t stride, int64_t rows, int64_t inner, const void* xq,
                          int64_t columns, float* y, int64_t ldy, const float* bias, const MatvecPlan& plan, float* partial,
                          uint32_t* counters, cudaStream_t s);

// ---- shards.cu -------------------------------------------------------------
cudaError_t launch_gather_shards(const float* src, int64_t shards, int64_t columns, int64_t shard_rows, float* dst,
                                 int64_t ldy, cudaStream_t s);

// ---- gemm.cu ---------------------------------------------------------------
struct GemmOperands {
    uint32_t type;        // kTypeQ8_0 or kTypeQ5_K
    int64_t M, N, K;      // activation rows, view rows (output columns), inner
    int64_t n_first;      // first weight row of the view (multiple of 4)
    // tensor maps: 0 weight operand, 1 activation operand, 2 weight scale
    // tile (Q8_0 one-hot scales / Q5_K min operand), 3 activation scale tile
    // (Q8_0 fp16 scales / Q8_K min operand), 4 Q5_K weight d, 5 Q5_K weight
    // dmin, 6 Q8_K activation d (unused entries may hold any valid map)
    CUtensorMap tm[7];
    CUtensorMap tm_y;     // output map (fp32 [M][ldy], box {32, 64}) when tma_store
    int tma_store;        // 1: write the output tile with TMA stores
    float* y;
    int64_t ldy;
    const float* bias;    // may be null (indexed by view-local column)
    float* dump;          // debug: raw per-item block dots, or null
    uint32_t* status;     // device status word
};
int gemm_smem_bytes();
cudaError_t launch_gemm(const GemmOperands& op, int num_sms, cudaStream_t s);

}  // namespace pxq
