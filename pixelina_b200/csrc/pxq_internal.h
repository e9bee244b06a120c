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
constexpr int kQ6KPadBytes = 224; // the same, padded to 16-byte multiples on the device (TMA rows)
constexpr uint32_t kTypeQ8_0 = 8;
constexpr uint32_t kTypeQ5_K = 13;
constexpr uint32_t kTypeQ6_K = 14;

// ---- quantize.cu -----------------------------------------------------------
// GGUF-format activation blocks (bit-exact with the reference quantizers).
cudaError_t launch_quantize_q8_0_blocks(const float* x, void* y, int64_t rows, int64_t inner, int64_t ldx, cudaStream_t s);
cudaError_t launch_quantize_q8_K_blocks(const float* x, void* y, int64_t rows, int64_t inner, int64_t ldx, cudaStream_t s);
// Tensor-core operand formats for the GEMM (same rounding, different layout):
//   Q8_0: xq [rows][inner]: the int8 quants themselves (kind 1) or as exact
//         fp16 values (kinds 0, 2); kinds 0, 1: dxT fp32 [inner/32][ldd], the
//         stored fp16 block scales as fp32, block-major; kind 2: the fp16
//         scales row-major [rows][ldd]
//   Q8_K: xq fp16 [rows][inner]: the int8 quants as exact fp16 values
//         dxT fp32 [inner/256][ldd]: per-block scale, block-major
//         amin fp16 [rows][inner/256*16]: split 32-element sums for the Q5_K
//         min term, (hi_j, lo_j) with bsum2_j = 64*hi_j + lo_j
cudaError_t launch_quantize_q8_0_operand(const float* x, void* xq, void* dx, int kind, int64_t rows, int64_t inner,
                                         int64_t ldx, int64_t ldd, cudaStream_t s);
cudaError_t launch_quantize_q8_K_operand(const float* x, __half* xq, float* dxT, __half* amin, int64_t rows, int64_t inner,
                                         int64_t ldx, int64_t ldd, cudaStream_t s);

// Q6_K weight rows padded for the device: 210-byte super-blocks -> 224.
cudaError_t launch_pad_q6_K(const void* src, void* dst, int64_t superblocks, cudaStream_t s);

// ---- repack.cu -------------------------------------------------------------
// One-time weight repack into the GEMM operand layout (bit-exact unpack).
// gate_rows = F > 0: a gated weight (F gate rows, then F up rows) packed as
// 128-row groups [64 gate rows j..j+63][the 64 matching up rows].
// Q8_0 (operand kind as in GemmOperands::q8_kind): wq [rows][inner] int8
// quants (kind 1) or their exact fp16 values (kinds 0, 2); kinds 0, 1: dT
// fp32 [inner/32][ldn] the fp16 block scales, block-major; kind 2: ws1h fp16
// [rows][inner/32*16], for block b a 16-wide group with the block's scale at
// position b % 16 and zeros elsewhere (the weight side of the tensor-core
// scale product).
cudaError_t launch_repack_q8_0(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, void* wq, float* dT,
                               __half* ws1h, int64_t ldn, int kind, int64_t gate_rows, cudaStream_t s);
cudaError_t launch_repack_q5_K(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, __half* wv, float* dT,
                               float* dminT, __half* bmin, int64_t ldn, int64_t gate_rows, cudaStream_t s);
// Q6_K: raw rows are the device's padded super-blocks (stride bytes per row).
cudaError_t launch_repack_q6_K(const uint8_t* raw, int64_t rows, int64_t inner, int64_t stride, __half* wab, float* dT,
                               int64_t ldn, int64_t gate_rows, cudaStream_t s);

// y[c*ldy + n] = silu(s[c*2F + n]) * s[c*2F + F + n] for c < columns, n < F:
// the gated epilogue after a matvec over a gated weight's 2F rows
// (tensor_silu then tensor_gate, src/tensor.cpp:199-208, :334-345).
cudaError_t launch_gate_rows(const float* s, int64_t columns, int64_t F, float* y, int64_t ldy, cudaStream_t st);

cudaError_t launch_decode(const uint8_t* data, uint32_t type, int64_t count, float* out, cudaStream_t s);

// ---- noalloc.cu ------------------------------------------------------------
// The static scratch array's device address on `device` (set up on first
// use, with that device current), or null; and clearing its counter region.
void* noalloc_scratch(int device);
cudaError_t noalloc_clear_counters(int device);

// ---- matvec.cu -------------------------------------------------------------
// y[c*ldy + r] = dot(W row r, X row c) for c < columns <= 8, raw GGUF weights.
//
// Q5_K: a persistent kernel over tiles of TR = 64, 32 or 16 weight rows, each
// tile's K range cut into stages of 128/TR super-blocks (22.5 KB), loaded by
// TMA through a tensor map over the raw weight bytes (64-bit elements, box
// {128/TR*176/8, TR}; the weight keeps one map per tile shape, index
// matvec_map_index(TR)).  Either every CTA owns whole tiles, or the flattened
// stage sequence is split evenly over the CTAs (stream-K) and a tile whose
// stages span several CTAs is finished, in fixed CTA order, by the last of
// them to arrive.  The activation is the matvec operand below (records of
// kQ8KMvBytes).
// Q8_0: 16-row groups, K split over `ks` CTAs per group when groups are few;
// the activation is GGUF Q8_0 blocks.
//
// One call's scratch (256-byte aligned, total_bytes): uint32 counters at
// off_counters = 0, in a region of at least kMvCounterRegion bytes that holds
// nothing else; the activation operand at off_act; fp32 partial sums at
// off_partial.  The counters must be zero when the matvec starts: the scratch
// starts zeroed, the quantize kernel of a call clears them, and every
// completed matvec leaves them zero again -- so a fused call (no quantize
// kernel) finds them zero whatever the previous call on the scratch was.
constexpr int kMvStageSuperBlocks = 8;                    // tile rows / 16 x super-blocks per stage
constexpr int kMvStageWeightBytes = 16 * kMvStageSuperBlocks * kQ5KBytes;  // 22528, any tile shape
constexpr int kMvTileShapes = 3;                         // 64 x 2, 32 x 4 and 16 x 8 super-blocks
constexpr int kQ8KMvBytes = 288;
constexpr int kQ80SbBytes = 8 * 34;                       // eight Q8_0 blocks (256 values) as stored
constexpr int kQ80MvBytes = 288;                          // Q8_0 matvec record: {i8 quants as kQ8KMvBytes; f32 d[8] at 256}
constexpr int kQ8KQ6Bytes = 304;                          // Q8_K record for Q6_K weights: {f32 d; pad; i8 qs[256] at 16; i16 bsums[16] at 272}
constexpr size_t kMvCounterRegion = 16 << 10;            // scratch bytes reserved for counters  // {i8 quants [4 pairs][4 lanes][2][8]; i16 32-element sums[8]; f32 d; pad}

struct MatvecPlan {
    uint32_t type = 0;
    int64_t rows = 0, inner = 0, columns = 0;
    int tile_rows = 64;                      // Q5_K: tile height
    int64_t tiles = 0, spt = 0, stages = 0;  // Q5_K: tiles, stages per tile, total stages
    int grid = 0;                            // CTAs
    int ks = 1, chunk = 0;                   // Q8_0: K slices per row group, blocks per slice
    int64_t rowgroups = 0;                   // Q8_0: 16-row groups
    bool streamed = false;                   // the TMA-fed kernel (K-quants; Q8_0 when inner % 256 == 0)
    bool fused = false;                      // streamed: the matvec quantizes the activation itself
    int64_t gated_half = 0;                  // K-quants, gated weight [gate; up]: F / 64 (the epilogue writes silu(g) * u)
    size_t act_bytes = 0, partial_bytes = 0, counter_bytes = 0;
    size_t off_counters = 0, off_act = 0, off_partial = 0, total_bytes = 0;
    // testing only (K-quants): CTA 0 loads nothing, so its bounded waits run
    // out and report a status, and the call's split-K counters are left the
    // way an interrupted call leaves them
    bool debug_stall = false;
};
// fuse_quantize: allow the plan to let the matvec quantize a small
// activation itself (then act_bytes is 0 and launch_matvec takes x).
// gated (K-quants, rows = 2F, F % 64 == 0): the weight is a gated pair [gate;
// up] and the matvec writes y[c][n] = silu(gate_n . x_c) * (up_n . x_c) for
// n < F, each CTA taking gate tile j and up tile j (64 rows each).
MatvecPlan plan_matvec(uint32_t type, int64_t rows, int64_t inner, int64_t columns, int num_sms, bool fuse_quantize = false,
                       bool gated = false);
int matvec_map_index(int tile_rows);
// Quantize the plan's `columns` activation rows (row stride ldx floats) into
// the operand at `act`; clears `counters` (plan.counter_bytes) when non-null.
// Launched with programmatic stream serialization.
cudaError_t launch_matvec_quantize(const MatvecPlan& plan, const float* x, int64_t ldx, void* act, uint32_t* counters,
                                   cudaStream_t s);
// The matvec.  Q5_K reads the weight through maps[matvec_map_index(tile
// rows)] (tensor maps over the whole weight) starting at row `row_first`; Q8_0 reads `w` (the view's first
// row).  Launched with programmatic stream serialization: the Q5_K kernel
// streams weights before the previous kernel of the stream has finished and
// touches every other buffer only after it.
cudaError_t launch_matvec(const MatvecPlan& plan, const CUtensorMap* maps, int64_t row_first, const uint8_t* w,
                          int64_t stride, const void* act, const float* x, int64_t ldx, float* y, int64_t ldy,
                          const float* bias, float* partial, uint32_t* counters, uint32_t* status, cudaStream_t s);

// Launch with programmatic stream serialization (see griddep_wait in
// pxq_device.cuh).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- attention.cu ----------------------------------------------------------
// fp32 multi-head attention with the semantics of tensor_attention
// (src/tensor.cpp:347-427): q/out [q_rows][heads*head_dim], k/v
// [k_rows][kv_heads*head_dim]; query ranges (host arrays, at most
// kAttnMaxRanges) give each row's permitted key prefix.  head_dim 64, 80 or
// 128.  q_rows <= 8 uses the key-split kernel and needs
// attention_scratch_bytes() of scratch.
constexpr int kAttnMaxRanges = 8;
size_t attention_scratch_bytes(int64_t q_rows, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t k_rows, int num_sms);
cudaError_t launch_attention(const float* q, int64_t q_rows, const float* k, const float* v, int64_t k_rows, int heads,
                             int kv_heads, int head_dim, const int64_t* range_end, const int64_t* range_keys,
                             const int* range_causal, int nranges, int64_t query_offset, float* out, float* scratch,
                             size_t scratch_bytes, int num_sms, cudaStream_t s);

// ---- shards.cu -------------------------------------------------------------
cudaError_t launch_gather_shards(const float* src, int64_t shards, int64_t columns, int64_t shard_rows, float* dst,
                                 int64_t ldy, cudaStream_t s);

// ---- gemm.cu ---------------------------------------------------------------
constexpr int kMaxScatter = 8;  // destinations of a scattering GEMM (one per rank of a node)

struct GemmOperands {
    uint32_t type;        // kTypeQ8_0, kTypeQ5_K or kTypeQ6_K
    int q8_kind;          // Q8_0 operand kind (gemm_q8.cu): 0 fp16 quants, scales applied on the CUDA cores;
                          // 1 int8 quants (kind::i8), scales on the CUDA cores; 2 fp16 quants, scale
                          // products from a one-hot tensor-core MMA; 3 kind 0's operands on CTA pairs;
                          // 4 int8 quants (kind::i8) with kind 2's scale products
    int64_t M, N, K;      // activation rows, view rows (output columns), inner
    int64_t n_first;      // first weight row of the view (multiple of 4)
    // tensor maps (boxes as listed in gemm.cu and gemm_q8.cu): 0 weight
    // operand, 1 activation operand, 2 Q5_K weight min operand, 3 Q8_K
    // activation min operand, 4 weight block scales (Q8_0 d / K-quant d),
    // 5 Q5_K weight dmin, 6 activation block scales (unused entries may hold
    // any valid map)
    CUtensorMap tm[7];
    CUtensorMap tm_y;     // output map (fp32 [M][ldy], box {32, gemm_store_rows}) when tma_store
    int tma_store;        // 1: write the output tile with TMA stores
    float* y;
    int64_t ldy;
    const float* bias;    // may be null (indexed by view-local column)
    float* dump;          // debug: raw per-item block dots, or null
    int gated;            // gated weight (2F interleaved rows, N = 2F): y[m][n < F] = silu(gate) * up
    uint32_t* status;     // device status word
    // scatter (ndst > 0): element (m, n), besides y[m * ldy + n], also goes to
    // ydst[k][m * ldy + col_off + n] for every k < ndst -- peers' buffers (P2P stores over NVLink)
    float* ydst[kMaxScatter];
    int ndst;
    int dst_vec4;         // every ydst[k] + col_off 16-byte aligned and ldy % 4 == 0
    int64_t col_off;
    // Q8_0 one-CTA kernels: the scatter as TMA stores (the output tile's staged
    // boxes also stored through tm_ydst[k], maps of ydst[k] + col_off shaped
    // like tm_y) instead of plain stores from the drain warps
    int tma_dst;
    CUtensorMap tm_ydst[kMaxScatter];
};
// Rows of one CTA's activation box in the GEMM's tensor maps (tmX, tmXs),
// and of a whole output tile (the activation scale map tmDx's box).
int gemm_activation_rows(uint32_t type);
int gemm_tile_activation_rows(uint32_t type);
// Activation rows of one output TMA store (the output map's box is {32, rows});
// 0 when the type's epilogue stores directly.
int gemm_store_rows(uint32_t type);
cudaError_t launch_gemm(const GemmOperands& op, int num_sms, cudaStream_t s);

// ---- gemm_q8.cu -------------------------------------------------------------
// The Q8_0 GEMM (called by launch_gemm).  32-blocks per fp32 scale box
// (operand kinds 0 and 1: 2 or 4).
cudaError_t launch_gemm_q8(const GemmOperands& op, int num_sms, cudaStream_t s);
int gemm_q8_scale_box(int kind);

}  // namespace pxq
