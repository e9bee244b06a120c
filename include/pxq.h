/*
 * pxq.h -- C ABI of the B200 quantized-matmul backend (libpxq.so).
 *
 * This is the drop-in boundary for Pixelina's quantized-matmul path.  Every
 * entry point uses plain pointers and sizes; "device" pointers are CUDA
 * device addresses on the current device, "host" pointers are ordinary (or
 * pinned) host memory.  Streams are passed as `void*` holding a cudaStream_t
 * (NULL = the legacy default stream).  All functions return PXQ_OK (0) or a
 * PXQ_ERR_* code; pxq_last_error() gives a one-line description for the
 * calling thread.
 *
 * Layout conventions follow the reference (paths are within the Pixelina
 * source tree):
 *   - "rows" = weight rows = output features (N), "columns" = activation rows
 *     (M), "inner" = K, exactly as in cpu_quant_matmul
 *     (src/kernels_quant.cpp:369).
 *   - weights are GGUF rows: rows x weight_bytes({inner}, type) bytes
 *     (src/model.cpp:87-121);
 *   - activations are row-major fp32 [columns][inner];
 *   - the output is row-major [columns][ldy]: output[c*ldy + r]
 *     (src/kernels_quant.cpp:396 has ldy == rows).
 */
#ifndef PXQ_H
#define PXQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PXQ_OK 0
#define PXQ_ERR_INVALID 1       /* bad argument (null pointer, zero size, ...) */
#define PXQ_ERR_UNSUPPORTED 2   /* type/shape this backend does not handle */
#define PXQ_ERR_CUDA 3          /* a CUDA runtime call failed */
#define PXQ_ERR_NO_MEMORY 4     /* device allocation failed */
#define PXQ_ERR_NO_DEVICE 5     /* no usable sm_100 device */
#define PXQ_ERR_DEVICE_STATUS 6 /* a kernel reported a bounded-wait timeout */
#define PXQ_ERR_IO 7            /* a model file could not be opened or mapped */
#define PXQ_ERR_FORMAT 8        /* a model file is not a GGUF v3 file this loader accepts */
#define PXQ_ERR_TIMEOUT 9       /* a multi-GPU set-up or collective did not complete in time (communicator aborted) */

/* GGML type ids, src/model_types.h:13-21 */
#define PXQ_TYPE_F32 0
#define PXQ_TYPE_F16 1
#define PXQ_TYPE_Q8_0 8
#define PXQ_TYPE_Q5_K 13
#define PXQ_TYPE_Q6_K 14
#define PXQ_TYPE_BF16 30

#if defined(__GNUC__)
#define PXQ_API __attribute__((visibility("default")))
#else
#define PXQ_API
#endif

typedef struct pxq_weight pxq_weight; /* opaque device-resident weight */

/* Library version, (major << 16) | minor. */
PXQ_API int pxq_version(void);

/* Description of the last error on the calling thread ("" if none). */
PXQ_API const char* pxq_last_error(void);

/* Select and initialise a CUDA device for the calling thread.  Replaces the
 * session start of the GPU backend (VulkanSession::initialize,
 * src/backend_vulkan.h:124-137).  Fails with PXQ_ERR_NO_DEVICE unless the
 * device is compute capability 10.x. */
PXQ_API int pxq_init(int device);

/* Bytes of a [inner, rows] tensor of `type`, 0 if invalid.  Same contract as
 * weight_bytes (src/model.cpp:87-121). */
PXQ_API uint64_t pxq_weight_bytes(uint64_t inner, uint64_t rows, uint32_t type);

/* fp32 device rows -> GGUF Q8_0 blocks on the device, bit-exact with
 * quantize_row_q8_0_ref (src/kernels_quant.cpp:120-144).
 * x: [rows][inner] fp32; blocks: rows * inner/32 * 34 bytes; inner % 32 == 0. */
PXQ_API int pxq_quantize_q8_0(const float* x, void* blocks, size_t rows, size_t inner, void* stream);

/* fp32 device rows -> Q8_K blocks (292 bytes per 256 values), bit-exact with
 * quantize_row_q8_K_ref (src/kernels_quant.cpp:80-118); inner % 256 == 0. */
PXQ_API int pxq_quantize_q8_K(const float* x, void* blocks, size_t rows, size_t inner, void* stream);

/* fp32 device rows -> the matvec's Q8_K records (PXQ_Q8K_MATVEC_BYTES per 256
 * values): the same quants and scale as pxq_quantize_q8_K, permuted for the
 * matvec's tensor-core fragments -- quants of sub-block j (32 values), elements
 * 8t..8t+7, at byte 64*(j/2) + 16*t + 8*(j%2) (t = 0..3) -- then the eight
 * 32-element sums bsums[2j] + bsums[2j+1] (int16) at byte 256 and d (fp32) at
 * byte 272.  The layout pxq_matvec feeds itself for Q5_K weights; exported so
 * it can be checked bit for bit.  inner % 256 == 0, rows <= 8. */
#define PXQ_Q8K_MATVEC_BYTES 288
PXQ_API int pxq_quantize_q8_K_matvec(const float* x, void* records, size_t rows, size_t inner, void* stream);

/* Dequantize `count` values of a Q8_0 / Q5_K / Q6_K device buffer to fp32,
 * bit-exact with cpu_decode (src/backend_cpu.cpp:24-101). */
PXQ_API int pxq_decode(const void* data, uint32_t type, size_t count, float* out, void* stream);

/* Make a weight device-resident.  `bytes` holds rows GGUF rows of `type`
 * (host memory if bytes_on_device == 0, else a device pointer that is
 * copied).  `key` (may be NULL) names the tensor; uploading the same key
 * again returns the cached weight, as the Vulkan weight cache does with
 * "file:name:offset:bytes" (src/backend_vulkan.cpp:742-758).
 * Supported types: Q8_0, Q5_K, Q6_K. */
PXQ_API int pxq_weight_upload(const void* bytes, int bytes_on_device, uint32_t type, size_t inner, size_t rows, const char* key,
                      pxq_weight** out);

/* Upload the gate and up projections of a gated feed-forward as one weight
 * for pxq_matmul_gated: `gate` and `up` each hold `rows` GGUF rows of `type`
 * (host or device, as for pxq_weight_upload).  The callers' pairs: separate
 * tensors (src/inference.cpp:331-332, src/qwen_vl.cpp:396) or the two row
 * slices of one fused tensor (src/qwen_image.cpp:271).  rows must be a
 * multiple of 64.  The weight serves pxq_matmul_gated only. */
PXQ_API int pxq_weight_upload_gated(const void* gate, const void* up, int bytes_on_device, uint32_t type, size_t inner,
                                    size_t rows, const char* key, pxq_weight** out);

/* Gated feed-forward projection in one call:
 *   output[c*ldy + r] = silu(g) * u,  g = input[c] . gate[r],  u = input[c] . up[r]
 * with silu(g) = g / (1 + exp(-g)) -- the callers' tensor_linear, tensor_linear,
 * tensor_silu, tensor_gate sequence (src/tensor.cpp:199-208, :334-345) with
 * no intermediate tensors.  columns <= 8 runs the matvec over both
 * projections and a small epilogue kernel; larger runs the tensor-core GEMM
 * with the gate applied in its epilogue. */
PXQ_API int pxq_matmul_gated(pxq_weight* w, const float* input, size_t columns, float* output, size_t ldy, void* stream);

/* Drop a weight (its device copies are freed once no call uses them). */
PXQ_API int pxq_weight_release(pxq_weight* w);

/* Drop every cached weight. */
PXQ_API int pxq_weight_cache_clear(void);

/* Residency budget of the weight cache on the current device, in bytes (the
 * Vulkan backend's cache_limit, src/backend_vulkan.cpp:421 and :1055).
 * Cached weights -- uploads with a key and the host-buffer drop-in's own
 * uploads -- count their device bytes against it: the raw rows plus the GEMM
 * operand copies.  When an upload or an operand copy would exceed it, the
 * least recently used entries give way (src/backend_vulkan.cpp:671-681,
 * :751): the drop-in's uploads whole (made again from the caller's bytes on
 * its next call), other cached weights their operand copies (rebuilt on the
 * next GEMM); weights in use by a call are skipped, and an upload goes ahead
 * when nothing is left to evict.  A cached upload larger than the whole
 * budget fails with PXQ_ERR_UNSUPPORTED (the reference returns nullptr, its
 * caller falls back).  Uploads without a key are the caller's and not
 * counted.  0 restores the default: 85 % of device memory less min(512 MiB,
 * a quarter of that). */
PXQ_API int pxq_weight_cache_limit(uint64_t bytes);
/* Cached bytes, budget and entries on the current device. */
PXQ_API int pxq_weight_cache_usage(uint64_t* bytes, uint64_t* limit, uint64_t* entries);

/* Device matmul through a weight: the operator behind cpu_matmul
 * (src/backend_cpu.cpp:103-133) and vulkan_matmul
 * (src/backend_vulkan.cpp:1083-1094).
 *   output[c*ldy + r] = sum_k input[c][k] * W[row_first + r][k]   (+ bias[r])
 * for c < columns, r < row_count.  row_first/row_count select a row range of
 * the weight like tensor_linear_rows (src/tensor.cpp:529-544); bias (device,
 * row_count floats, may be NULL) is added as tensor_linear does
 * (src/tensor.cpp:162-170).  input, output, bias are device pointers.
 * columns <= 8 runs the streaming matvec, larger runs the tensor-core GEMM. */
PXQ_API int pxq_matmul(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
               size_t ldy, const float* bias, void* stream);

/* pxq_matmul forced onto the small-M matvec kernel (columns <= 8), the
 * GPU counterpart of shaders/matvec.comp's role (src/backend_vulkan.cpp:887). */
PXQ_API int pxq_matvec(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
               size_t ldy, const float* bias, void* stream);

/* pxq_matmul forced onto the tensor-core GEMM (any columns >= 1), the
 * counterpart of shaders/quantize.comp + shaders/matmul_mmq.comp
 * (src/backend_vulkan.cpp:963-981). */
PXQ_API int pxq_gemm(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
             size_t ldy, const float* bias, void* stream);

/* Host-buffer drop-in for cpu_quant_matmul (src/kernels_quant.cpp:369-412,
 * declared src/tensor.h:74): same arguments, same output layout
 * output[c*rows + r].  Weights are cached on the device by host address,
 * shape, type and a fingerprint of the bytes (the first and last 256 bytes
 * and 256 samples of 16 bytes), so a buffer freed and refilled at the same
 * address is uploaded again; the entries live in the weight cache
 * (pxq_weight_cache_limit).  The input is copied to the device and the
 * output back before the call returns.  Returns PXQ_OK when handled, PXQ_ERR_UNSUPPORTED exactly
 * where the reference returns false (unsupported type, zero sizes,
 * inner % block != 0, inner > INT32_MAX). */
PXQ_API int pxq_quant_matmul(const unsigned char* weights, uint32_t type, const float* input, float* output, size_t rows,
                     size_t columns, size_t inner);

/* pxq_matmul with HOST input and output buffers through a device-resident
 * weight: the input is copied to the device, the product computed there and
 * the output copied back before the call returns (what cpu_matmul's callers
 * expect, src/backend_cpu.cpp:103-133).  Uses a per-thread stream. */
PXQ_API int pxq_matmul_host(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns,
                            float* output, size_t ldy);

/* Wait for `stream` and report any bounded-wait timeout a kernel recorded
 * since the last call (PXQ_ERR_DEVICE_STATUS), then clear it.  On that
 * error it also waits for the whole device and zeroes the split-K counters
 * of every matvec scratch on it (the per-stream buffers and the
 * no-allocation array), which an interrupted matvec may leave non-zero;
 * later calls then compute correctly again. */
PXQ_API int pxq_synchronize(void* stream);

/* Reorder all-gathered output shards into one row-major output: src holds
 * `shards` consecutive [columns][shard_rows] blocks (what an all-gather of
 * per-rank outputs produces), dst is [columns][ldy] with shard s at column
 * offset s*shard_rows.  Device pointers.  The layout step of the N-sharded
 * multi-GPU matmul (no counterpart in the single-process reference). */
PXQ_API int pxq_gather_shards(const float* src, size_t shards, size_t columns, size_t shard_rows, float* dst, size_t ldy,
                      void* stream);

/* The N-sharded multi-GPU matmul in one kernel: this rank's weight rows
 * [row_first, row_first + row_count) times `input` (columns > 8: the GEMM
 * path), with element (m, n) stored into dsts[k][m * ldy + col_offset + n]
 * for every k < ndst: dsts[0] is this GPU's own output (written like any
 * output), dsts[1..] the other ranks' outputs (device pointers opened with
 * pxq_ipc_open), written by the GEMM epilogue over NVLink from the same
 * staged tiles while the next tiles compute.  Replaces the matmul, the
 * all-gather and pxq_gather_shards of the N-sharded path (each rank holding
 * weight rows of cpu_quant_matmul's independent output columns,
 * src/kernels_quant.cpp:390-398).  The caller orders the ranks around the
 * call (every rank's buffers free before, a barrier after).  1 <= ndst <= 8. */
PXQ_API int pxq_matmul_scatter(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns,
                               float* const* dsts, size_t ndst, size_t ldy, size_t col_offset, void* stream);

/* Device buffers other processes of the node can map (CUDA IPC): allocate
 * `bytes` on the current device and write its PXQ_IPC_HANDLE_BYTES handle;
 * open another process's handle as a pointer usable in this process's
 * kernels (peer access over NVLink); close / free them. */
#define PXQ_IPC_HANDLE_BYTES 64
PXQ_API int pxq_ipc_alloc(size_t bytes, void** ptr, void* handle);
PXQ_API int pxq_ipc_free(void* ptr);
PXQ_API int pxq_ipc_open(const void* handle, void** ptr);
PXQ_API int pxq_ipc_close(void* ptr);

/* ---- N-sharded multi-GPU matmul (one process per GPU, NCCL) ---------------
 * No counterpart in the single-process reference: its CPU path computes all
 * output columns of cpu_quant_matmul in one process
 * (src/kernels_quant.cpp:389-400).  Output columns (weight rows) are
 * independent, so G ranks each hold an even share of the weight rows --
 * rank r the rows [r*N/G, (r+1)*N/G), uploaded as an ordinary pxq_weight --
 * compute their columns for the replicated activation, and assemble the
 * full row-major output on every rank, bit-identical to one GPU.
 *
 * Failure handling: the communicator is created non-blocking and every wait
 * (set-up, collectives, synchronize) polls NCCL's asynchronous error state
 * against the communicator's timeout; on expiry it is aborted and the call
 * returns PXQ_ERR_TIMEOUT (a rank that never joins or never reaches a
 * collective).  An aborted communicator fails every later call; destroy it
 * and create a new one. */
typedef struct pxq_comm pxq_comm;
typedef struct pxq_sharded_out pxq_sharded_out;
#define PXQ_COMM_ID_BYTES 128

/* One rank (usually rank 0) creates the communicator id and hands its
 * PXQ_COMM_ID_BYTES bytes to every rank by any channel (ncclGetUniqueId). */
PXQ_API int pxq_comm_unique_id(void* id);

/* Join communicator `id` as `rank` of `world` (1..8) on the calling thread's
 * current device (select it with pxq_init first).  Returns PXQ_ERR_TIMEOUT
 * if not every rank joined within timeout_ms. */
PXQ_API int pxq_comm_init(const void* id, int world, int rank, int timeout_ms, pxq_comm** out);
PXQ_API int pxq_comm_size(const pxq_comm* comm, int* world, int* rank);
/* Host-side barrier of all ranks (bounded by the timeout). */
PXQ_API int pxq_comm_barrier(pxq_comm* comm);
/* Wait for `stream` (bounded by the timeout; NCCL errors abort the
 * communicator), then report kernel status like pxq_synchronize. */
PXQ_API int pxq_comm_synchronize(pxq_comm* comm, void* stream);
PXQ_API int pxq_comm_destroy(pxq_comm* comm);

/* Collective: an fp32 output [columns][ldy] on every rank, each rank's
 * buffer mapped into every other rank's address space (CUDA IPC handles
 * exchanged over the communicator).  *local (may be NULL) receives this
 * rank's buffer (device pointer).  Destroy collectively too. */
PXQ_API int pxq_sharded_output_create(pxq_comm* comm, size_t columns, size_t ldy, pxq_sharded_out** out, float** local);
PXQ_API int pxq_sharded_output_destroy(pxq_sharded_out* out);

/* Y = input * W^T with W's N = G*shard_rows rows split over the ranks;
 * `shard` holds this rank's shard_rows rows.  input: device fp32
 * [columns][inner], replicated on every rank.  Every rank calls it with the
 * same shapes, in the same order.  Queued on `stream`; complete after
 * pxq_comm_synchronize.
 *   out != NULL (columns > 8): fused -- the GEMM epilogue stores its
 *     columns into every rank's `out` buffer over NVLink while later tiles
 *     compute, between two device-side barriers; Y is in each rank's local
 *     buffer (`output`, `ldy` unused).
 *   out == NULL: the rank's columns go to stream-ordered scratch, an NCCL
 *     all-gather collects every rank's block and one re-layout kernel
 *     writes `output` (device [columns][ldy], ldy >= N). */
PXQ_API int pxq_sharded_matmul(pxq_comm* comm, pxq_weight* shard, size_t shard_rows, const float* input, size_t columns,
                               pxq_sharded_out* out, float* output, size_t ldy, void* stream);

/* The same with host buffers, the multi-GPU counterpart of pxq_quant_matmul:
 * the host input [columns][inner] is copied to this rank's device, the fused
 * sharded product computed, and the full output [columns][N] copied back to
 * the host before the call returns.  Output buffers are created on the
 * first call of a shape (collectively) and kept for later calls. */
PXQ_API int pxq_sharded_matmul_host(pxq_comm* comm, pxq_weight* shard, size_t shard_rows, const float* input, size_t columns,
                                    size_t inner, float* output);

/* ---- quantize once, multiply many ----------------------------------------
 * The reference quantizes the activation inside every cpu_quant_matmul call
 * (src/kernels_quant.cpp:382-388).  These entry points split that step out so
 * one quantized activation can feed several weights with the same inner size
 * (q/k/v, gate/up) and so the two kernels can be timed separately.  The
 * activation is quantized in the format the given weight type needs (Q8_0
 * blocks for Q8_0 weights, Q8_K for K-quants), bit-exact as above. */
typedef struct pxq_activation pxq_activation;

/* Quantize device fp32 [columns][inner] for weights of `weight_type`. */
PXQ_API int pxq_activation_quantize(uint32_t weight_type, const float* input, size_t columns, size_t inner,
                                    pxq_activation** out, void* stream);

/* pxq_matmul on an already-quantized activation. */
PXQ_API int pxq_matmul_quantized(pxq_weight* w, size_t row_first, size_t row_count, const pxq_activation* a,
                                 float* output, size_t ldy, const float* bias, void* stream);

/* Free an activation once the work queued on `stream` that reads it is done. */
PXQ_API int pxq_activation_release(pxq_activation* a, void* stream);

/* Number of CUDA kernels this library has launched in this process (all
 * devices).  Lets a caller check that its work ran on the GPU path. */
PXQ_API uint64_t pxq_kernel_launches(void);

/* ---- decode matvec without device allocation --------------------------------
 * No counterpart in the reference (its CPU path allocates its quantized
 * activations with std::vector on every call).  For callers that must not
 * allocate device memory while they run -- a decode loop that cannot stall on
 * the allocator, a region where the application forbids cudaMalloc, an
 * embedder with a fixed device-memory budget: same contract and results as
 * pxq_matvec (columns 1..8), but the quantized activation rows go to a
 * static device array of PXQ_NOALLOC_SCRATCH_BYTES owned by this library
 * (held on every device that loads it, until exit) instead of freshly
 * allocated scratch.  The array holds the matvec's counters (16 KiB), the
 * quantized activation rows (columns * inner/256 * 288 bytes for Q5_K and
 * for Q8_0 when inner % 256 == 0, columns * inner/32 * 34 + 64 for other
 * Q8_0, columns * inner/256 * 304 for Q6_K;
 * none when the matvec quantizes a small activation itself) and its fp32
 * partial sums (up to 2 * columns * 256 bytes per CTA, about 1.2 MB for 8
 * columns on a 148-SM GPU); a call whose total exceeds
 * PXQ_NOALLOC_SCRATCH_BYTES is rejected with PXQ_ERR_UNSUPPORTED before any
 * work is queued.
 * The weight must already be uploaded and the current device must be the
 * weight's.  The first call on a device looks up the array's device address
 * (one-time set-up); make that call before any stream capture.  All calls on
 * a device share the array: calls whose GPU work may overlap (unordered
 * streams) race, so order them. */
#define PXQ_NOALLOC_SCRATCH_BYTES (4 << 20)

PXQ_API int pxq_matvec_noalloc(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns,
                               float* output, size_t ldy, const float* bias, void* stream);

/* Testing the failure path: a K-quant matvec of the whole weight (columns
 * 1..8) in which CTA 0 loads nothing, so its bounded waits run out after
 * their limit (about 2 s) and record a status, and its split-K counters are
 * left the way an interrupted call leaves them -- in the stream's scratch
 * (static_scratch == 0) or in the no-allocation array (1).  The output is
 * not meaningful.  pxq_synchronize then returns PXQ_ERR_DEVICE_STATUS and
 * restores the scratch.  Nothing faults or hangs: every wait is bounded. */
PXQ_API int pxq_debug_matvec_stall(pxq_weight* w, const float* input, size_t columns, float* output, int static_scratch,
                                   void* stream);

/* Debug/parity: run the tensor-core GEMM but store, instead of the scaled
 * sum, every exact block dot it computed.  dump (device) receives
 * items x columns x row_count floats, item-major; items = inner/32 for Q8_0,
 * 5*inner/256 for Q5_K (per super-block: four 64-value sums of sc*q5*q8,
 * then the min sum of m*bsum) and 4*inner/256 for Q6_K (per super-block:
 * four 64-value sums of sc*(q6-32)*q8).  These are the int32 block dots of
 * pix_dot_q8_0 / pix_dot_q5_K / pix_dot_q6_K (src/kernels_quant.cpp:339-365,
 * :163-254, :256-337), exact as floats. */
PXQ_API int pxq_gemm_block_dots(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* dump,
                        void* stream);

/* ---- attention: the callers' step after the quantized linears --------- */

/* A query range of tensor_attention's second overload (PixAttentionRange,
 * src/tensor.h:58-63): rows [query_begin, query_end) may attend to keys
 * [0, key_end), further limited to key <= query_offset + row when causal. */
typedef struct {
    size_t query_begin, query_end, key_end;
    int causal;
} pxq_attention_range;

/* Multi-head softmax attention in fp32 with the semantics of
 * tensor_attention (src/tensor.cpp:347-427): q and output [q_rows][heads *
 * head_dim], k and v [k_rows][kv_heads * head_dim] (device, row-major),
 * kv head of head h = h / (heads / kv_heads), scores scaled by
 * 1/sqrt(head_dim).  ranges: 1..8 contiguous ranges covering [0, q_rows)
 * (NULL with nranges 0: one range with key_end = k_rows, causal = 0 -- the
 * first overload's non-causal case; its causal case is one range with
 * causal = 1 and query_offset 0).  head_dim 64, 80 or 128. */
PXQ_API int pxq_attention(const float* q, size_t q_rows, const float* k, const float* v, size_t k_rows, size_t heads,
                          size_t kv_heads, size_t head_dim, const pxq_attention_range* ranges, size_t nranges,
                          size_t query_offset, float* output, void* stream);

/* ---- GGUF model files: the format step in front of the upload ---------- */

/* A GGUF v3 file mapped read-only, its tensor directory parsed with the
 * acceptance rules of Pixelina's loader (PixModelFile::open,
 * src/model.cpp:138-251). */
typedef struct pxq_gguf pxq_gguf;

/* One tensor of the directory (PixWeight, src/model.h:33-39). */
typedef struct {
    const char* name;    /* valid while the file is open */
    uint32_t type;       /* GGML type id (PXQ_TYPE_*) */
    uint32_t rank;       /* 1..5 */
    uint64_t shape[5];   /* GGML order: shape[0] is contiguous (inner) */
    uint64_t offset;     /* absolute byte offset of the tensor data in the file */
    uint64_t bytes;      /* storage bytes */
} pxq_gguf_tensor;

/* Open and parse; PXQ_ERR_IO when the file cannot be opened or mapped,
 * PXQ_ERR_FORMAT where the reference's loader returns MODEL_ERROR_FORMAT. */
PXQ_API int pxq_gguf_open(const char* path, pxq_gguf** out);
PXQ_API int pxq_gguf_close(pxq_gguf* f);
PXQ_API size_t pxq_gguf_tensor_count(const pxq_gguf* f);
PXQ_API size_t pxq_gguf_metadata_count(const pxq_gguf* f);
/* The mapped file (tensor bytes at data + offset). */
PXQ_API const void* pxq_gguf_data(const pxq_gguf* f);
/* Tensor `index` in name order (the reference's std::map order). */
PXQ_API int pxq_gguf_tensor_at(const pxq_gguf* f, size_t index, pxq_gguf_tensor* out);
PXQ_API int pxq_gguf_find(const pxq_gguf* f, const char* name, pxq_gguf_tensor* out);

/* Upload rows [row_first, row_first + row_count) of a Q8_0 / Q5_K / Q6_K
 * tensor (row_count 0: to the end) through pxq_weight_upload, cached under
 * "file:name:offset:bytes" of the row range -- the Vulkan backend's weight
 * cache identity (src/backend_vulkan.cpp:742-758), which also gives
 * tensor_linear_rows views (src/tensor.cpp:529-544) their own entry. */
PXQ_API int pxq_gguf_upload(pxq_gguf* f, const char* name, size_t row_first, size_t row_count, pxq_weight** out);

/* Upload a gated pair for pxq_matmul_gated: `rows` rows of tensor `gate`
 * from gate_first and of tensor `up` from up_first (the same tensor for the
 * DiT's fused gate/up, src/qwen_image.cpp:271). */
PXQ_API int pxq_gguf_upload_gated(pxq_gguf* f, const char* gate, size_t gate_first, const char* up, size_t up_first,
                                  size_t rows, pxq_weight** out);

#ifdef __cplusplus
}
#endif

#endif /* PXQ_H */
