// api.cu -- host side of the C ABI declared in include/pxq.h.
//
// Responsibilities:
//   * device context per CUDA device (SM count, kernel status word, the
//     cuTensorMapEncodeTiled entry point fetched through the runtime);
//   * the device weight cache: raw GGUF rows uploaded once, plus a lazily
//     built GEMM operand copy (repack.cu), keyed like the Vulkan backend's
//     cache (src/backend_vulkan.cpp:742-758);
//   * dispatch of a matmul to the streaming matvec (columns <= 8) or the
//     tensor-core GEMM; the matvec's scratch is a buffer kept per (device,
//     stream) so a steady decode loop allocates nothing, the GEMM's comes
//     from the stream-ordered allocator;
//   * the host-buffer cpu_quant_matmul drop-in.
// There is no CPU compute path here: an unsupported case is reported as an
// error status (the reference's `false`), never computed on the host.
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <list>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "pxq.h"
#include "pxq_internal.h"

using namespace pxq;

namespace {

thread_local std::string t_error;

int fail(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_error = buf;
    return code;
}

#define PXQ_CUDA(call)                                                                                 \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess) return fail(PXQ_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceCtx {
    bool ready = false;
    int sms = 0;
    uint32_t* status = nullptr;  // device word written by kernels on a bounded-wait timeout
    EncodeTiledFn encode = nullptr;
    // weight cache residency (guarded by g_mutex): the device bytes of cached
    // weights (raw rows + GEMM operand copies) and their budget
    uint64_t cache_bytes = 0;
    uint64_t cache_limit = 0;
    uint64_t cache_default = 0;
};

constexpr int kMaxDevices = 16;
std::mutex g_mutex;
DeviceCtx g_dev[kMaxDevices];
thread_local int t_device = -1;

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

int init_device(int device)
{
    if (device < 0 || device >= kMaxDevices) return fail(PXQ_ERR_NO_DEVICE, "device %d out of range", device);
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count)
        return fail(PXQ_ERR_NO_DEVICE, "no CUDA device %d (found %d)", device, count);
    PXQ_CUDA(cudaSetDevice(device));
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceCtx& d = g_dev[device];
    if (!d.ready) {
        cudaDeviceProp prop;
        PXQ_CUDA(cudaGetDeviceProperties(&prop, device));
        if (prop.major != 10)
            return fail(PXQ_ERR_NO_DEVICE, "device %d is sm_%d%d; this build targets sm_100a", device, prop.major, prop.minor);
        d.sms = prop.multiProcessorCount;
        // the weight cache's default budget, as the Vulkan backend sizes its
        // cache_limit: 85 % of device memory less a reserve of min(512 MiB, a
        // quarter) for activations and scratch (src/backend_vulkan.cpp:417-421)
        const uint64_t heap = (uint64_t)((double)prop.totalGlobalMem * 0.85);
        const uint64_t reserve = std::min<uint64_t>((uint64_t)512 << 20, heap / 4);
        d.cache_default = d.cache_limit = heap - reserve;
        PXQ_CUDA(cudaMalloc(&d.status, 256));
        PXQ_CUDA(cudaMemset(d.status, 0, 256));
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        PXQ_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) return fail(PXQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        d.encode = reinterpret_cast<EncodeTiledFn>(fn);
        // keep stream-ordered scratch cached between calls
        cudaMemPool_t pool;
        PXQ_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
        uint64_t threshold = UINT64_MAX;
        PXQ_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold));
        d.ready = true;
    }
    t_device = device;
    return PXQ_OK;
}

int ensure_device(DeviceCtx** out)
{
    if (t_device < 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
        int rc = init_device(dev);
        if (rc) return rc;
    } else {
        int cur = -1;
        cudaGetDevice(&cur);
        if (cur != t_device) PXQ_CUDA(cudaSetDevice(t_device));
    }
    *out = &g_dev[t_device];
    return PXQ_OK;
}

int make_map(const DeviceCtx* d, CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
             uint64_t stride1_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw)
{
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = d->encode(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(PXQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu box %u x %u", (int)r,
                    (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)stride1_bytes, b0, b1);
    return PXQ_OK;
}

// 3-D tiled map: dims {d0, d1, d2}, byte strides {s1, s2}, box {b0, b1, b2}.
int make_map3(const DeviceCtx* d, CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
              uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2)
{
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {s1, s2};
    const cuuint32_t box[3] = {b0, b1, b2};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = d->encode(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(PXQ_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d): dims %llu x %llu x %llu box %u x %u x %u", (int)r,
                    (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, b0, b1, b2);
    return PXQ_OK;
}

// GEMM operand copy of (a row range of) a weight.
struct Packed {
    int64_t rows = 0;   // packed rows
    int64_t ldn = 0;    // row stride of the K-quant scale planes
    void* mem = nullptr;
    uint64_t bytes = 0;       // device bytes of `mem`
    void* wv = nullptr;       // operand [rows][K]: fp16 (Q6_K: [rows][2K], even and parity planes) or Q8_0 int8
    __half* ws = nullptr;     // Q5_K min operand [rows][nsb*16]
    float* d = nullptr;       // block scales: Q8_0 d [K/32][ldn], Q5_K / Q6_K d [nsb][ldn]
    int q8_kind = 0;          // Q8_0: int8 operand (kind::i8 GEMM)
    float* dmin = nullptr;    // Q5_K dmin [nsb][ldn]
    CUtensorMap tmW, tmWs, tmD, tmDm;
    ~Packed()
    {
        if (mem) cudaFree(mem);
    }
};

}  // namespace

struct pxq_weight {
    uint32_t type = 0;
    int64_t inner = 0, rows = 0, stride = 0;
    // gated: rows = 2F, the gate projection's F rows then the up projection's
    // F rows (pxq_weight_upload_gated); only pxq_matmul_gated takes it
    bool gated = false;
    int device = 0;
    uint8_t* raw = nullptr;
    CUtensorMap mv_map[kMvTileShapes];  // Q5_K: raw bytes as u64 [rows][stride/8], the matvec's TMA views
    std::string key;
    std::unique_ptr<Packed> packed;                       // whole tensor
    std::map<std::pair<int64_t, int64_t>, std::unique_ptr<Packed>> views;  // unaligned row views
    // weight cache (guarded by g_mutex): a keyed weight counts its device
    // bytes against the device's budget; `internal` ones (the host-buffer
    // drop-in's own uploads) may be evicted whole, any cached weight may lose
    // its operand copies (rebuilt on the next GEMM); `pins` counts the calls
    // using the weight right now, which nothing evicts under
    uint64_t raw_bytes = 0;
    bool cached = false, internal = false;
    uint64_t last_use = 0;
    int pins = 0;
    uint64_t packed_bytes() const
    {
        uint64_t b = packed ? packed->bytes : 0;
        for (const auto& kv : views) b += kv.second->bytes;
        return b;
    }
    ~pxq_weight()
    {
        if (raw) cudaFree(raw);
    }
};

// A quantized activation: the matvec operand (columns <= 8: Q8_0 blocks, or
// the Q8_K matvec records) or the tensor-core operand layout (GEMM), in one
// stream-ordered allocation.
struct pxq_activation {
    uint32_t wtype = 0;     // weight type it was quantized for
    int64_t M = 0, K = 0;
    bool blocks = false;    // true: matvec operand; false: GEMM operand
    void* mem = nullptr;
    void* xq = nullptr;     // operand: the quants [M][K], exact fp16 values (Q8_0: or int8)
    void* scale = nullptr;  // operand: fp32 block scales, block-major [K/block][ldd]
    int q8_kind = 0;        // Q8_0: int8 operand
    __half* amin = nullptr; // operand (Q8_K): min-term split sums [M][nsb*16]
    int64_t ldd = 0;
    CUtensorMap tmX, tmXs, tmDx;
};

namespace pxq {
cudaError_t matvec_fused(const pxq_weight* w, size_t row_first, size_t row_count, const float* input, float* output,
                         size_t ldy, const float* bias, const MatvecPlan& plan, uint8_t* scratch, uint32_t* status,
                         cudaStream_t s);
}

namespace {

std::unordered_map<std::string, pxq_weight*> g_cache;  // guarded by g_mutex

// Q8_0 GEMM operand kind (gemm_q8.cu): 0 = exact fp16 copies of the quants
// (kind::f16) with the scales applied on the CUDA cores, 1 = the int8 quants
// (kind::i8) likewise, 2 = fp16 copies with the scale products from a
// one-hot tensor-core MMA, 3 = kind 0's operands on CTA pairs (256 x 256
// tiles), 4 = kind 2 with the int8 quants (kind::i8 block dots).  Read once
// from PXQ_Q8_0_MMA ("f16", "i8", "f16s", "pair", "i8s"); the default is
// kind 2, the fastest measured (its drain converts nothing: the kind::f16
// block dots arrive in TMEM as fp32, where kind 4's int32 dots cost one
// int-to-float conversion per element and block).
int q8_operand_kind()
{
    static const int v = [] {
        const char* e = getenv("PXQ_Q8_0_MMA");
        if (e && strcmp(e, "f16") == 0) return 0;
        if (e && strcmp(e, "i8") == 0) return 1;
        if (e && strcmp(e, "pair") == 0) return 3;
        if (e && strcmp(e, "i8s") == 0) return 4;
        return 2;
    }();
    return v;
}
std::atomic<uint64_t> g_launches{0};

cudaError_t counted(cudaError_t e, uint64_t n = 1)
{
    if (e == cudaSuccess) g_launches.fetch_add(n, std::memory_order_relaxed);
    return e;
}

// 64-bit FNV-1a over the first and last 256 bytes and 256 samples of 16
// bytes spread over the buffer: the host-buffer drop-in's cache identity.
uint64_t fingerprint(const void* data, uint64_t n)
{
    const uint8_t* p = static_cast<const uint8_t*>(data);
    uint64_t h = 1469598103934665603ull ^ n;
    auto mix = [&](uint64_t off, uint64_t len) {
        for (uint64_t i = 0; i < len && off + i < n; i++) {
            h ^= p[off + i];
            h *= 1099511628211ull;
        }
    };
    mix(0, 256);
    if (n > 256) mix(n - 256, 256);
    for (uint64_t k = 0; k < 256; k++) mix(n / 256 * k, 16);
    return h;
}

// ---- weight cache residency (the Vulkan backend's weight cache,
// src/backend_vulkan.cpp:671-681 evict, :742-758 weight) ---------------------
std::atomic<uint64_t> g_use_clock{0};

// Drop a cached weight's bytes from its device's count and forget it.
// g_mutex held; the caller frees the weight.
void uncache(pxq_weight* w)
{
    if (!w->cached) return;
    DeviceCtx& d = g_dev[w->device];
    d.cache_bytes -= w->raw_bytes + w->packed_bytes();
    auto it = g_cache.find(w->key);
    if (it != g_cache.end() && it->second == w) g_cache.erase(it);
    w->cached = false;
}

// Evict, least recently used first, until `need` more bytes fit the budget
// of `device`: internal weights (the host-buffer drop-in's uploads, re-made
// from the caller's bytes on the next call) whole, other cached weights
// their GEMM operand copies (rebuilt on the next GEMM).  Weights in use
// (pins) and `keep` are skipped.  g_mutex held.  Like the Vulkan backend,
// an upload still goes ahead when nothing is left to evict.
void make_room(int device, uint64_t need, const pxq_weight* keep)
{
    DeviceCtx& d = g_dev[device];
    bool synced = false;
    while (d.cache_bytes + need > d.cache_limit) {
        pxq_weight* victim = nullptr;
        for (auto& kv : g_cache) {
            pxq_weight* w = kv.second;
            if (w->device != device || w == keep || w->pins) continue;
            if (!w->internal && !w->packed_bytes()) continue;
            if (!victim || w->last_use < victim->last_use) victim = w;
        }
        if (!victim) return;
        if (!synced) {
            cudaDeviceSynchronize();  // no kernel still reads what is freed
            synced = true;
        }
        if (victim->internal) {
            uncache(victim);
            delete victim;
        } else {
            d.cache_bytes -= victim->packed_bytes();
            victim->packed.reset();
            victim->views.clear();
        }
    }
}

// A weight used by a call: most recently used, and not evicted until the call
// has queued its work.
struct Pin {
    pxq_weight* w;
    explicit Pin(pxq_weight* w_) : w(w_)
    {
        if (!w) return;
        std::lock_guard<std::mutex> lock(g_mutex);
        w->pins++;
        w->last_use = ++g_use_clock;
    }
    ~Pin()
    {
        if (!w) return;
        std::lock_guard<std::mutex> lock(g_mutex);
        w->pins--;
    }
};

int build_packed(const DeviceCtx* d, pxq_weight* w, int64_t first, int64_t count, std::unique_ptr<Packed>& out,
                 cudaStream_t s)
{
    auto pk = std::make_unique<Packed>();
    const int64_t K = w->inner;
    const bool q5 = w->type == kTypeQ5_K, q6 = w->type == kTypeQ6_K, q8 = w->type == kTypeQ8_0;
    const int kind = q8 ? q8_operand_kind() : 0;
    const bool i8 = kind == 1 || kind == 4, onehot = q8 && (kind == 2 || kind == 4);
    const int64_t nb = (q5 || q6) ? K / kQKK : K / kQK8_0;
    const int64_t Kop = q6 ? 2 * K : K;  // Q6_K: even and parity planes per chunk
    const int64_t elem = i8 ? 1 : 2;
    pk->rows = count;
    pk->ldn = round_up(count, 4);
    pk->q8_kind = kind;
    const size_t wv_bytes = (size_t)count * Kop * elem;
    const size_t ws_bytes = (q5 || onehot) ? (size_t)count * nb * 32 : 0;
    const size_t s_bytes = onehot ? 0 : (size_t)nb * pk->ldn * 4;
    const size_t dm_bytes = q5 ? s_bytes : 0;
    const size_t off_ws = round_up((int64_t)wv_bytes, 1024);
    const size_t off_d = off_ws + round_up((int64_t)ws_bytes, 1024);
    const size_t off_dm = off_d + round_up((int64_t)s_bytes, 1024);
    const size_t total = off_dm + round_up((int64_t)dm_bytes, 1024) + 1024;
    if (w->cached) make_room(w->device, total, w);
    if (cudaMalloc(&pk->mem, total) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_NO_MEMORY, "cannot allocate %zu bytes for the GEMM operand copy", total);
    }
    pk->bytes = total;
    if (w->cached) g_dev[w->device].cache_bytes += total;
    uint8_t* base = static_cast<uint8_t*>(pk->mem);
    pk->wv = base;
    pk->ws = reinterpret_cast<__half*>(base + off_ws);
    pk->d = reinterpret_cast<float*>(base + off_d);
    pk->dmin = reinterpret_cast<float*>(base + off_dm);
    PXQ_CUDA(cudaMemsetAsync(pk->mem, 0, total, s));
    const uint8_t* src = w->raw + first * w->stride;
    const int64_t gate_rows = w->gated ? w->rows / 2 : 0;  // whole-tensor copies only (first = 0)
    if (q6) {
        PXQ_CUDA(counted(launch_repack_q6_K(src, count, K, w->stride, static_cast<__half*>(pk->wv), pk->d, pk->ldn, gate_rows, s)));
    } else if (q8) {
        PXQ_CUDA(counted(launch_repack_q8_0(src, count, K, w->stride, pk->wv, pk->d, pk->ws, pk->ldn, kind, gate_rows, s)));
    } else {
        PXQ_CUDA(counted(launch_repack_q5_K(src, count, K, w->stride, static_cast<__half*>(pk->wv), pk->d, pk->dmin, pk->ws,
                                            pk->ldn, gate_rows, s)));
    }
    // operand box: one 128-byte swizzle row (64 fp16 or 128 int8) x 128 rows
    int rc = make_map(d, &pk->tmW, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pk->wv, Kop, count,
                      Kop * elem, (uint32_t)(128 / elem), 128, CU_TENSOR_MAP_SWIZZLE_128B);
    // unused maps of a type hold the weight map (any valid map will do)
    pk->tmWs = pk->tmD = pk->tmDm = pk->tmW;
    if (!rc && (q5 || onehot))
        rc = make_map(d, &pk->tmWs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pk->ws, nb * 16, count, nb * 32, 16, 128,
                      CU_TENSOR_MAP_SWIZZLE_32B);
    if (!rc && !onehot)
        rc = make_map(d, &pk->tmD, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pk->d, count, nb, pk->ldn * 4, 128,
                      q8 ? (uint32_t)gemm_q8_scale_box(kind) : 1u, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc && q5)
        rc = make_map(d, &pk->tmDm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pk->dmin, count, nb, pk->ldn * 4, 128, 1,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    out = std::move(pk);
    return PXQ_OK;
}

// Operand copy covering [first, first+count): the whole-tensor copy when the
// view starts on a 4-row boundary (TMA coordinates of fp32 scale planes must
// be 16-byte aligned), otherwise a dedicated copy of just the view.
int get_packed(const DeviceCtx* d, pxq_weight* w, int64_t first, int64_t count, const Packed** pk, int64_t* n_first,
               cudaStream_t s)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    if (first % 4 == 0) {
        if (!w->packed) {
            int rc = build_packed(d, w, 0, w->rows, w->packed, s);
            if (rc) return rc;
        }
        *pk = w->packed.get();
        *n_first = first;
        return PXQ_OK;
    }
    auto key = std::make_pair(first, count);
    auto it = w->views.find(key);
    if (it == w->views.end()) {
        std::unique_ptr<Packed> p;
        int rc = build_packed(d, w, first, count, p, s);
        if (rc) return rc;
        it = w->views.emplace(key, std::move(p)).first;
    }
    *pk = it->second.get();
    *n_first = 0;
    return PXQ_OK;
}

int check_matmul_args(pxq_weight* w, size_t row_first, size_t row_count, const void* input, size_t columns, const void* output,
                      size_t ldy)
{
    if (!w || !input || !output) return fail(PXQ_ERR_INVALID, "null weight, input or output");
    if (w->gated) return fail(PXQ_ERR_INVALID, "gated weight: use pxq_matmul_gated");
    if (!columns || !row_count) return fail(PXQ_ERR_INVALID, "zero columns or rows");
    if (row_first > (size_t)w->rows || row_count > (size_t)w->rows - row_first)
        return fail(PXQ_ERR_INVALID, "row range [%zu, %zu) outside weight with %lld rows", row_first, row_first + row_count,
                    (long long)w->rows);
    if (ldy < row_count && columns > 1) return fail(PXQ_ERR_INVALID, "ldy %zu < row_count %zu", ldy, row_count);
    if (w->type != kTypeQ8_0 && w->type != kTypeQ5_K && w->type != kTypeQ6_K)
        return fail(PXQ_ERR_UNSUPPORTED, "weight type %u not supported", w->type);
    return PXQ_OK;
}

// layout: 0 = by batch size (blocks for M <= 8), 1 = GGUF blocks, 2 = GEMM operand
int quantize_activation(DeviceCtx* d, uint32_t wtype, const float* input, int64_t M, int64_t K, int layout,
                        pxq_activation** out, cudaStream_t s)
{
    *out = nullptr;
    if (!input || !M || !K) return fail(PXQ_ERR_INVALID, "null input or zero size");
    if (wtype != kTypeQ8_0 && wtype != kTypeQ5_K && wtype != kTypeQ6_K)
        return fail(PXQ_ERR_UNSUPPORTED, "weight type %u not supported", wtype);
    const bool q5 = wtype != kTypeQ8_0;  // K-quants: Q8_K activations
    if (K % (q5 ? kQKK : kQK8_0)) return fail(PXQ_ERR_UNSUPPORTED, "inner %lld not a multiple of the block", (long long)K);
    auto a = std::make_unique<pxq_activation>();
    a->wtype = wtype;
    a->M = M;
    a->K = K;
    a->blocks = layout == 0 ? (M <= 8) : (layout == 1);
    const int64_t nb = q5 ? K / kQKK : K / kQK8_0;
    cudaError_t e;
    if (a->blocks) {
        const MatvecPlan plan = plan_matvec(wtype, 1, K, M, d->sms);
        if (cudaMallocAsync(&a->mem, plan.act_bytes, s) != cudaSuccess) {
            cudaGetLastError();
            return fail(PXQ_ERR_NO_MEMORY, "scratch allocation of %zu bytes failed", plan.act_bytes);
        }
        e = launch_matvec_quantize(plan, input, K, a->mem, nullptr, s);
    } else {
        const int kind = q5 ? 0 : q8_operand_kind();
        const bool i8 = kind == 1 || kind == 4, onehot = !q5 && (kind == 2 || kind == 4);
        a->q8_kind = kind;
        // scales: fp32 block-major [nb][round_up(M, 4)], or (one-hot kind) fp16
        // row-major [M][round_up(nb, 8)]
        a->ldd = onehot ? round_up(nb, 8) : round_up(M, 4);
        const size_t xq_bytes = (size_t)M * K * (i8 ? 1 : 2);
        const size_t sc_bytes = onehot ? (size_t)M * a->ldd * 2 : (size_t)nb * a->ldd * 4;
        const size_t amin_bytes = q5 ? (size_t)M * nb * 32 : 0;
        const size_t off_sc = round_up((int64_t)xq_bytes, 1024);
        const size_t off_amin = off_sc + round_up((int64_t)sc_bytes, 1024);
        const size_t total = off_amin + round_up((int64_t)amin_bytes, 1024) + 1024;
        if (cudaMallocAsync(&a->mem, total, s) != cudaSuccess) {
            cudaGetLastError();
            return fail(PXQ_ERR_NO_MEMORY, "scratch allocation of %zu bytes failed", total);
        }
        uint8_t* base = static_cast<uint8_t*>(a->mem);
        a->xq = base;
        a->scale = base + off_sc;
        a->amin = reinterpret_cast<__half*>(base + off_amin);
        e = q5 ? launch_quantize_q8_K_operand(input, static_cast<__half*>(a->xq), static_cast<float*>(a->scale), a->amin, M, K, K,
                                              a->ldd, s)
               : launch_quantize_q8_0_operand(input, a->xq, a->scale, kind, M, K, K, a->ldd, s);
        const uint32_t xr = (uint32_t)gemm_activation_rows(wtype);  // one CTA's rows of an output tile
        const int64_t elem = i8 ? 1 : 2;
        int rc = make_map(d, &a->tmX, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a->xq, K, M, K * elem,
                          (uint32_t)(128 / elem), xr, CU_TENSOR_MAP_SWIZZLE_128B);
        if (!rc && q5) {
            rc = make_map(d, &a->tmXs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a->amin, nb * 16, M, nb * 32, 16, xr,
                          CU_TENSOR_MAP_SWIZZLE_32B);
            if (!rc) rc = make_map(d, &a->tmDx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a->scale, M, nb, a->ldd * 4,
                                   (uint32_t)gemm_tile_activation_rows(wtype), 1,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
        } else if (!rc && onehot) {
            rc = make_map(d, &a->tmXs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a->scale, nb, M, a->ldd * 2, 16, xr,
                          CU_TENSOR_MAP_SWIZZLE_32B);
            a->tmDx = a->tmX;
        } else if (!rc) {
            a->tmXs = a->tmX;
            // the drain's activation scales: a whole output tile's rows (kind 3: a CTA pair's 256)
            const uint32_t tile_rows = kind == 3 ? 256u : (uint32_t)gemm_tile_activation_rows(wtype);
            rc = make_map(d, &a->tmDx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a->scale, M, nb, a->ldd * 4, tile_rows,
                          (uint32_t)gemm_q8_scale_box(kind), CU_TENSOR_MAP_SWIZZLE_NONE);
        }
        if (rc) {
            cudaFreeAsync(a->mem, s);
            return rc;
        }
    }
    if (counted(e) != cudaSuccess) {
        cudaFreeAsync(a->mem, s);
        return fail(PXQ_ERR_CUDA, "quantize launch failed: %s", cudaGetErrorString(e));
    }
    *out = a.release();
    return PXQ_OK;
}

void free_activation(pxq_activation* a, cudaStream_t s)
{
    if (!a) return;
    if (a->mem) cudaFreeAsync(a->mem, s);
    delete a;
}

// Matvec of a pre-quantized activation: partial sums and counters from the
// stream-ordered allocator, counters cleared by a memset.
int run_matvec(DeviceCtx* d, pxq_weight* w, size_t row_first, size_t row_count, const pxq_activation* a, float* output,
               size_t ldy, const float* bias, cudaStream_t s)
{
    if (!a->blocks) return fail(PXQ_ERR_UNSUPPORTED, "matvec handles at most 8 columns (got %lld)", (long long)a->M);
    const MatvecPlan plan = plan_matvec(w->type, (int64_t)row_count, w->inner, a->M, d->sms);
    // counters and partial sums of this call; its activation region stays unused
    void* ws = nullptr;
    float* partial = nullptr;
    uint32_t* counters = nullptr;
    if (plan.counter_bytes || plan.partial_bytes) {
        if (cudaMallocAsync(&ws, plan.total_bytes, s) != cudaSuccess) {
            cudaGetLastError();
            return fail(PXQ_ERR_NO_MEMORY, "matvec workspace allocation failed");
        }
        partial = plan.partial_bytes ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + plan.off_partial) : nullptr;
        counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + plan.off_counters);
        if (plan.counter_bytes) PXQ_CUDA(cudaMemsetAsync(counters, 0, plan.counter_bytes, s));
    }
    cudaError_t e = launch_matvec(plan, w->mv_map, (int64_t)row_first, w->raw + row_first * w->stride, w->stride, a->mem,
                                  nullptr, 0, output, (int64_t)ldy, bias, partial, counters, d->status, s);
    if (ws) cudaFreeAsync(ws, s);
    if (counted(e) != cudaSuccess) return fail(PXQ_ERR_CUDA, "matvec launch failed: %s", cudaGetErrorString(e));
    return PXQ_OK;
}

// Scratch kept per (device, stream) for the fused quantize + matvec, so that
// a steady decode loop makes no allocation (and no allocator node separates
// its kernels in a captured graph).  Work on one stream is ordered, so one
// buffer per stream is race-free.  A buffer is only replaced when a call
// needs more; the old one is kept for the life of the process because a
// captured graph may still name it.
struct StreamScratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};
std::map<std::pair<int, cudaStream_t>, StreamScratch> g_stream_scratch;  // guarded by g_mutex
std::vector<void*> g_retired_scratch;                                     // guarded by g_mutex

// Zero the counter region of every matvec scratch on `device`: the
// per-stream buffers (current and retired) and the no-allocation array.  The
// caller has synchronized the device.
void reset_scratch_counters(int device)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    for (auto& kv : g_stream_scratch)
        if (kv.first.first == device && kv.second.ptr) cudaMemset(kv.second.ptr, 0, kMvCounterRegion);
    for (void* p : g_retired_scratch) cudaMemset(p, 0, kMvCounterRegion);
    noalloc_clear_counters(device);
}

// The stream's scratch (at least `need` bytes), or null when no device memory
// is left.  Growing it during a stream capture is allowed: like PyTorch's
// allocator, the cudaMalloc runs with this thread's capture mode relaxed, so
// the buffer outlives the graph and no allocator node enters it.
void* stream_scratch(int device, cudaStream_t s, size_t need)
{
    std::lock_guard<std::mutex> lock(g_mutex);
    StreamScratch& e = g_stream_scratch[{device, s}];
    if (e.bytes >= need) return e.ptr;
    size_t bytes = need > 2 * e.bytes ? need : 2 * e.bytes;
    if (bytes < ((size_t)4 << 20)) bytes = (size_t)4 << 20;
    bytes = (bytes + ((size_t)1 << 20) - 1) & ~(((size_t)1 << 20) - 1);
    void* p = nullptr;
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    const cudaError_t err = cudaMalloc(&p, bytes);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    // counters in the scratch must start at zero (calls leave them zero)
    if (cudaMemsetAsync(p, 0, bytes, s) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return nullptr;
    }
    if (e.ptr) g_retired_scratch.push_back(e.ptr);
    e.ptr = p;
    e.bytes = bytes;
    return p;
}

int run_gemm(DeviceCtx* d, pxq_weight* w, size_t row_first, size_t row_count, const pxq_activation* a, float* output,
             size_t ldy, const float* bias, float* dump, cudaStream_t s, float* const* dsts = nullptr, int ndst = 0,
             int64_t col_off = 0)
{
    if (a->blocks) return fail(PXQ_ERR_UNSUPPORTED, "activation was quantized for the matvec path");
    const Packed* pk = nullptr;
    int64_t n_first = 0;
    int rc = get_packed(d, w, (int64_t)row_first, (int64_t)row_count, &pk, &n_first, s);
    if (rc) return rc;
    if (w->type == kTypeQ8_0 && pk->q8_kind != a->q8_kind)
        return fail(PXQ_ERR_INVALID, "Q8_0 weight and activation operands were built for different MMA kinds");
    GemmOperands op;
    std::memset(&op, 0, sizeof(op));
    op.type = w->type;
    op.q8_kind = pk->q8_kind;
    op.M = a->M;
    op.N = (int64_t)row_count;
    op.K = a->K;
    op.n_first = n_first;
    op.y = output;
    op.ldy = (int64_t)ldy;
    op.bias = bias;
    op.dump = dump;
    op.status = d->status;
    op.gated = w->gated ? 1 : 0;
    op.ndst = ndst;
    op.col_off = col_off;
    op.dst_vec4 = ldy % 4 == 0 ? 1 : 0;
    for (int k = 0; k < ndst; k++) {
        op.ydst[k] = dsts[k];
        if ((reinterpret_cast<uintptr_t>(dsts[k] + col_off) & 15u) != 0) op.dst_vec4 = 0;
    }
    op.tm[0] = pk->tmW;
    op.tm[1] = a->tmX;
    op.tm[2] = pk->tmWs;
    op.tm[3] = a->tmXs;
    op.tm[4] = pk->tmD;
    op.tm[5] = pk->tmDm;
    op.tm[6] = a->tmDx;
    // TMA-store epilogue when output rows start 16-byte aligned and the row
    // length is a whole number of 16-byte units (a bulk tensor store clips the
    // innermost dimension only at 16-byte granularity)
    op.tma_store = 0;
    op.tm_y = op.tm[0];
    if (!dump && !w->gated && gemm_store_rows(w->type) > 0 && (reinterpret_cast<uintptr_t>(output) & 15u) == 0 &&
        (ldy % 4) == 0 && (row_count % 4) == 0) {
        if (make_map(d, &op.tm_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, output, row_count, (uint64_t)a->M, ldy * 4, 32,
                     (uint32_t)gemm_store_rows(w->type),
                     CU_TENSOR_MAP_SWIZZLE_NONE) == PXQ_OK)
            op.tma_store = 1;
        else
            op.tm_y = op.tm[0];
    }
    // scatter through TMA stores too where the destinations allow the same
    // boxes as the local output (Q8_0 one-CTA kernels)
    if (op.tma_store && ndst > 0 && op.dst_vec4 && w->type == kTypeQ8_0 && op.q8_kind != 3) {
        op.tma_dst = 1;
        for (int k = 0; k < ndst && op.tma_dst; k++)
            if (make_map(d, &op.tm_ydst[k], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dsts[k] + col_off, row_count, (uint64_t)a->M,
                         ldy * 4, 32, (uint32_t)gemm_store_rows(w->type), CU_TENSOR_MAP_SWIZZLE_NONE) != PXQ_OK)
                op.tma_dst = 0;
    }
    cudaError_t e = launch_gemm(op, d->sms, s);
    if (counted(e) != cudaSuccess) return fail(PXQ_ERR_CUDA, "gemm launch failed: %s", cudaGetErrorString(e));
    return PXQ_OK;
}

int check_activation(pxq_weight* w, const pxq_activation* a)
{
    if (!a) return fail(PXQ_ERR_INVALID, "null activation");
    if (a->wtype != w->type) return fail(PXQ_ERR_INVALID, "activation quantized for type %u, weight is %u", a->wtype, w->type);
    if (a->K != w->inner) return fail(PXQ_ERR_INVALID, "activation inner %lld != weight inner %lld", (long long)a->K,
                                      (long long)w->inner);
    return PXQ_OK;
}

// quantize + multiply + free, all stream-ordered; force: 0 auto, 1 matvec, 2 gemm
int run_matmul(DeviceCtx* d, pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns,
               float* output, size_t ldy, const float* bias, float* dump, int force, cudaStream_t s)
{
    if (force == 1 && columns > 8) return fail(PXQ_ERR_UNSUPPORTED, "matvec handles at most 8 columns (got %zu)", columns);
    if (w->type == kTypeQ8_0 || w->type == kTypeQ5_K) {
        if (w->inner % 8) return fail(PXQ_ERR_UNSUPPORTED, "inner %lld not a multiple of 8", (long long)w->inner);
    }
    if (force == 1 || (force == 0 && columns <= 8)) {
        if (!input) return fail(PXQ_ERR_INVALID, "null input");
        const MatvecPlan plan = plan_matvec(w->type, (int64_t)row_count, w->inner, (int64_t)columns, d->sms, true);
        void* scratch = stream_scratch(t_device, s, plan.total_bytes);
        const bool own = scratch == nullptr;
        if (own && cudaMallocAsync(&scratch, plan.total_bytes, s) != cudaSuccess) {
            cudaGetLastError();
            return fail(PXQ_ERR_NO_MEMORY, "matvec scratch allocation of %zu bytes failed", plan.total_bytes);
        }
        if (own && plan.fused && plan.counter_bytes)  // fresh memory: no quantize kernel clears the counters
            PXQ_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(scratch) + plan.off_counters, 0, plan.counter_bytes, s));
        cudaError_t e = matvec_fused(w, row_first, row_count, input, output, ldy, bias, plan, static_cast<uint8_t*>(scratch),
                                     d->status, s);
        if (own) cudaFreeAsync(scratch, s);
        if (e != cudaSuccess) return fail(PXQ_ERR_CUDA, "matvec launch failed: %s", cudaGetErrorString(e));
        return PXQ_OK;
    }
    pxq_activation* a = nullptr;
    int rc = quantize_activation(d, w->type, input, (int64_t)columns, w->inner, force, &a, s);
    if (rc) return rc;
    rc = run_gemm(d, w, row_first, row_count, a, output, ldy, bias, dump, s);
    free_activation(a, s);
    return rc;
}

}  // namespace

namespace pxq {
// Quantize + matvec with all scratch in `scratch` (plan.total_bytes, 256-byte
// aligned): the quantize kernel clears the counters, both kernels are
// launched with programmatic stream serialization.
cudaError_t matvec_fused(const pxq_weight* w, size_t row_first, size_t row_count, const float* input, float* output,
                         size_t ldy, const float* bias, const MatvecPlan& plan, uint8_t* scratch, uint32_t* status,
                         cudaStream_t s)
{
    float* partial = plan.partial_bytes ? reinterpret_cast<float*>(scratch + plan.off_partial) : nullptr;
    uint32_t* counters = plan.counter_bytes ? reinterpret_cast<uint32_t*>(scratch + plan.off_counters) : nullptr;
    cudaError_t e = cudaSuccess;
    uint8_t* act = scratch + plan.off_act;
    if (!plan.fused) e = counted(launch_matvec_quantize(plan, input, w->inner, act, counters, s));
    if (e == cudaSuccess)
        e = counted(launch_matvec(plan, w->mv_map, (int64_t)row_first, w->raw + row_first * w->stride, w->stride, act, input,
                                  w->inner, output, (int64_t)ldy, bias, partial, counters, status, s));
    return e;
}

// Read-only view of a weight handle (used by noalloc.cu).
int device_sm_count(int device) { return (device >= 0 && device < kMaxDevices && g_dev[device].ready) ? g_dev[device].sms : 148; }
uint32_t* device_status(int device) { return (device >= 0 && device < kMaxDevices && g_dev[device].ready) ? g_dev[device].status : nullptr; }

bool weight_view(const pxq_weight* w, uint32_t* type, int64_t* inner, int64_t* rows, int64_t* stride, const uint8_t** raw,
                 int* device)
{
    if (!w || w->gated) return false;
    *type = w->type;
    *inner = w->inner;
    *rows = w->rows;
    *stride = w->stride;
    *raw = w->raw;
    *device = w->device;
    return true;
}

// Set the calling thread's pxq_last_error() message.  Capacity for messages
// is reserved on first use so later error reports reuse it.
void record_error(const char* msg)
{
    if (t_error.capacity() < 512) t_error.reserve(512);
    t_error.assign(msg);
}
}  // namespace pxq

namespace {

// per-thread stream for the host-buffer entry point (the reference's session
// is thread-local too, src/backend_vulkan.cpp:86)
thread_local cudaStream_t t_stream = nullptr;
thread_local cudaStream_t t_up = nullptr, t_down = nullptr;  // host-buffer path: uploads, downloads
thread_local int t_stream_device = -1;

}  // namespace

extern "C" {

int pxq_version(void) { return (0 << 16) | 1; }

const char* pxq_last_error(void) { return t_error.c_str(); }

int pxq_init(int device)
{
    t_error.clear();
    return init_device(device);
}

uint64_t pxq_weight_bytes(uint64_t inner, uint64_t rows, uint32_t type)
{
    uint64_t block = 1, bytes;
    switch (type) {
    case PXQ_TYPE_F32: bytes = 4; break;
    case PXQ_TYPE_F16:
    case PXQ_TYPE_BF16: bytes = 2; break;
    case PXQ_TYPE_Q8_0: block = 32; bytes = 34; break;
    case PXQ_TYPE_Q5_K: block = 256; bytes = 176; break;
    case PXQ_TYPE_Q6_K: block = 256; bytes = 210; break;
    default: return 0;
    }
    if (!inner || inner % block || !rows) return 0;
    uint64_t count = inner / block;
    if (count > UINT64_MAX / rows) return 0;
    count *= rows;
    if (count > UINT64_MAX / bytes) return 0;
    return count * bytes;
}

int pxq_quantize_q8_0(const float* x, void* blocks, size_t rows, size_t inner, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!x || !blocks || !rows || !inner) return fail(PXQ_ERR_INVALID, "null pointer or zero size");
    if (inner % 32) return fail(PXQ_ERR_UNSUPPORTED, "inner %zu not a multiple of 32", inner);
    PXQ_CUDA(counted(launch_quantize_q8_0_blocks(x, blocks, rows, inner, inner, static_cast<cudaStream_t>(stream))));
    return PXQ_OK;
}

int pxq_quantize_q8_K(const float* x, void* blocks, size_t rows, size_t inner, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!x || !blocks || !rows || !inner) return fail(PXQ_ERR_INVALID, "null pointer or zero size");
    if (inner % 256) return fail(PXQ_ERR_UNSUPPORTED, "inner %zu not a multiple of 256", inner);
    PXQ_CUDA(counted(launch_quantize_q8_K_blocks(x, blocks, rows, inner, inner, static_cast<cudaStream_t>(stream))));
    return PXQ_OK;
}

int pxq_quantize_q8_K_matvec(const float* x, void* records, size_t rows, size_t inner, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!x || !records || !rows || !inner) return fail(PXQ_ERR_INVALID, "null pointer or zero size");
    if (inner % kQKK) return fail(PXQ_ERR_UNSUPPORTED, "inner %zu not a multiple of 256", inner);
    if (rows > 8) return fail(PXQ_ERR_UNSUPPORTED, "the matvec operand holds at most 8 rows (got %zu)", rows);
    static_assert(PXQ_Q8K_MATVEC_BYTES == kQ8KMvBytes, "record size");
    const MatvecPlan plan = plan_matvec(kTypeQ5_K, 1, (int64_t)inner, (int64_t)rows, d->sms);
    PXQ_CUDA(counted(launch_matvec_quantize(plan, x, (int64_t)inner, records, nullptr, static_cast<cudaStream_t>(stream))));
    return PXQ_OK;
}

int pxq_decode(const void* data, uint32_t type, size_t count, float* out, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!data || !out || !count) return fail(PXQ_ERR_INVALID, "null pointer or zero size");
    if (type != PXQ_TYPE_Q8_0 && type != PXQ_TYPE_Q5_K && type != PXQ_TYPE_Q6_K)
        return fail(PXQ_ERR_UNSUPPORTED, "decode of type %u not supported", type);
    if (count % (type == PXQ_TYPE_Q8_0 ? 32 : 256)) return fail(PXQ_ERR_INVALID, "count %zu not a whole number of blocks", count);
    PXQ_CUDA(counted(launch_decode(static_cast<const uint8_t*>(data), type, (int64_t)count, out, static_cast<cudaStream_t>(stream))));
    return PXQ_OK;
}

}  // extern "C"

namespace {

// Copy `count` raw GGUF rows (host or device bytes) into rows [first,
// first+count) of w's device copy; Q6_K super-blocks are padded to 224 bytes.
int copy_rows(pxq_weight* w, const void* bytes, int bytes_on_device, int64_t first, int64_t count)
{
    const uint64_t total = pxq_weight_bytes((uint64_t)w->inner, (uint64_t)count, w->type);
    uint8_t* dst = w->raw + first * w->stride;
    if (w->type != PXQ_TYPE_Q6_K) {
        PXQ_CUDA(cudaMemcpy(dst, bytes, total, bytes_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
        return PXQ_OK;
    }
    const void* src = bytes;
    void* tmp = nullptr;
    if (!bytes_on_device || (reinterpret_cast<uintptr_t>(bytes) & 1u)) {
        if (cudaMalloc(&tmp, total) != cudaSuccess) {
            cudaGetLastError();
            return fail(PXQ_ERR_NO_MEMORY, "cannot allocate %llu bytes of upload staging", (unsigned long long)total);
        }
        const cudaError_t e = cudaMemcpy(tmp, bytes, total, bytes_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(tmp);
            return fail(PXQ_ERR_CUDA, "weight copy failed: %s", cudaGetErrorString(e));
        }
        src = tmp;
    }
    cudaError_t e = launch_pad_q6_K(src, dst, (int64_t)(w->inner / 256 * count), nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) return fail(PXQ_ERR_CUDA, "Q6_K padding failed: %s", cudaGetErrorString(e));
    return PXQ_OK;
}

// Upload one weight from `parts` sources of `rows` rows each (one plain
// weight, or the gate and up projections of a gated weight, stacked).
int create_weight(DeviceCtx* d, const void* const* parts, int nparts, int bytes_on_device, uint32_t type, size_t inner,
                  size_t rows, const char* key, pxq_weight** out)
{
    *out = nullptr;
    if (type != PXQ_TYPE_Q8_0 && type != PXQ_TYPE_Q5_K && type != PXQ_TYPE_Q6_K)
        return fail(PXQ_ERR_UNSUPPORTED, "weight type %u not supported", type);
    const uint64_t total = pxq_weight_bytes(inner, rows, type);
    if (!total) return fail(PXQ_ERR_INVALID, "invalid weight shape [%zu, %zu] for type %u", inner, rows, type);
    if (inner > 0x7fffffffu || rows * nparts > 0x7fffffffu)
        return fail(PXQ_ERR_UNSUPPORTED, "weight shape [%zu, %zu] exceeds INT32_MAX", inner, rows);
    std::string k = key ? std::string(key) : std::string();
    const bool q6t = type == PXQ_TYPE_Q6_K;
    const uint64_t stride_dev = q6t ? (uint64_t)(inner / 256) * kQ6KPadBytes : pxq_weight_bytes(inner, 1, type);
    const uint64_t raw_need = stride_dev * (uint64_t)(rows * nparts) + 64;
    if (!k.empty()) {
        std::lock_guard<std::mutex> lock(g_mutex);
        auto it = g_cache.find(k);
        if (it != g_cache.end() && it->second->device == t_device) {
            if (it->second->gated != (nparts == 2))
                return fail(PXQ_ERR_INVALID, "cached weight \"%s\" was uploaded %s gated", k.c_str(), nparts == 2 ? "not" : "as");
            it->second->last_use = ++g_use_clock;
            *out = it->second;
            return PXQ_OK;
        }
        // a tensor larger than the whole budget is not cached: the reference's
        // "return nullptr" (src/backend_vulkan.cpp:750), the caller falls back
        if (raw_need > d->cache_limit)
            return fail(PXQ_ERR_UNSUPPORTED, "weight of %llu bytes exceeds the weight cache budget of %llu bytes",
                        (unsigned long long)raw_need, (unsigned long long)d->cache_limit);
        make_room(t_device, raw_need, nullptr);
    }
    auto w = std::make_unique<pxq_weight>();
    w->type = type;
    w->inner = (int64_t)inner;
    w->rows = (int64_t)(rows * nparts);
    w->gated = nparts == 2;
    w->stride = (int64_t)pxq_weight_bytes(inner, 1, type);
    w->device = t_device;
    w->key = k;
    const bool q6 = type == PXQ_TYPE_Q6_K;
    const uint64_t nsb = inner / 256;
    // Q6_K rows live on the device with every 210-byte super-block padded to
    // 224 bytes (16-byte multiples, as TMA rows need)
    if (q6) w->stride = (int64_t)(nsb * kQ6KPadBytes);
    const uint64_t dev_bytes = (uint64_t)w->stride * (uint64_t)w->rows;
    if (cudaMalloc(&w->raw, dev_bytes + 64) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_NO_MEMORY, "cannot allocate %llu bytes for weight", (unsigned long long)dev_bytes);
    }
    PXQ_CUDA(cudaMemset(w->raw + dev_bytes, 0, 64));
    for (int i = 0; i < nparts; i++)
        if (int rc = copy_rows(w.get(), parts[i], bytes_on_device, (int64_t)(i * rows), (int64_t)rows)) return rc;
    const uint64_t all_rows = (uint64_t)w->rows;
    std::memset(w->mv_map, 0, sizeof(w->mv_map));
    const bool q8_streamed = type == PXQ_TYPE_Q8_0 && inner % 256 == 0;
    if (type == PXQ_TYPE_Q5_K || q6 || q8_streamed) {
        // the matvec's TMA views, one box = one stage of a tr-row tile
        // (kMvStageSuperBlocks*16/tr super-blocks): Q5_K 64-row stages as a
        // 2-D view (rows of stride/8 64-bit words), the others as a 3-D view
        // (super-block, row, super-block words) that lands super-block-major;
        // a Q8_0 "super-block" is eight raw blocks (272 bytes)
        const uint32_t sbb = q6 ? kQ6KPadBytes : q8_streamed ? kQ80SbBytes : kQ5KBytes;
        if (type == PXQ_TYPE_Q5_K) {
            if (int rc = make_map(d, &w->mv_map[matvec_map_index(64)], CU_TENSOR_MAP_DATA_TYPE_UINT64, w->raw,
                                  (uint64_t)w->stride / 8, all_rows, (uint64_t)w->stride,
                                  (uint32_t)(kMvStageSuperBlocks / 4 * kQ5KBytes / 8), 64, CU_TENSOR_MAP_SWIZZLE_NONE))
                return rc;
        }
        for (int tr : {64, 32, 16}) {
            if (tr == 64 && type == PXQ_TYPE_Q5_K) continue;
            if (int rc = make_map3(d, &w->mv_map[matvec_map_index(tr)], CU_TENSOR_MAP_DATA_TYPE_UINT64, w->raw, sbb / 8,
                                   all_rows, nsb, (uint64_t)w->stride, sbb, sbb / 8, (uint32_t)tr,
                                   (uint32_t)(kMvStageSuperBlocks * 16 / tr)))
                return rc;
        }
    }
    w->raw_bytes = raw_need;
    if (!k.empty()) {
        std::lock_guard<std::mutex> lock(g_mutex);
        auto it = g_cache.find(k);
        if (it != g_cache.end()) {
            // another thread cached the same key meanwhile: keep that one
            // (the new copy is freed when `w` goes out of scope)
            *out = it->second;
            return PXQ_OK;
        }
        w->cached = true;
        w->last_use = ++g_use_clock;
        g_dev[t_device].cache_bytes += raw_need;
        g_cache[k] = w.get();
    }
    *out = w.release();
    return PXQ_OK;
}

}  // namespace

extern "C" {

int pxq_weight_upload(const void* bytes, int bytes_on_device, uint32_t type, size_t inner, size_t rows, const char* key,
                      pxq_weight** out)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!bytes || !out) return fail(PXQ_ERR_INVALID, "null bytes or out");
    const void* parts[1] = {bytes};
    return create_weight(d, parts, 1, bytes_on_device, type, inner, rows, key, out);
}

int pxq_weight_upload_gated(const void* gate, const void* up, int bytes_on_device, uint32_t type, size_t inner, size_t rows,
                            const char* key, pxq_weight** out)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!gate || !up || !out) return fail(PXQ_ERR_INVALID, "null gate, up or out");
    if (rows % 64) return fail(PXQ_ERR_UNSUPPORTED, "gated weights need a multiple of 64 rows (got %zu)", rows);
    const void* parts[2] = {gate, up};
    return create_weight(d, parts, 2, bytes_on_device, type, inner, rows, key, out);
}

int pxq_weight_release(pxq_weight* w)
{
    if (!w) return fail(PXQ_ERR_INVALID, "null weight");
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        uncache(w);
    }
    cudaDeviceSynchronize();
    delete w;
    return PXQ_OK;
}

int pxq_weight_cache_clear(void)
{
    std::vector<pxq_weight*> victims;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        for (auto& kv : g_cache) victims.push_back(kv.second);
        for (pxq_weight* w : victims) uncache(w);
    }
    cudaDeviceSynchronize();
    for (pxq_weight* w : victims) delete w;
    return PXQ_OK;
}

int pxq_weight_cache_limit(uint64_t bytes)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    std::lock_guard<std::mutex> lock(g_mutex);
    d->cache_limit = bytes ? bytes : d->cache_default;
    make_room(t_device, 0, nullptr);
    return PXQ_OK;
}

int pxq_weight_cache_usage(uint64_t* bytes, uint64_t* limit, uint64_t* entries)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    std::lock_guard<std::mutex> lock(g_mutex);
    uint64_t n = 0;
    for (auto& kv : g_cache)
        if (kv.second->device == t_device) n++;
    if (bytes) *bytes = d->cache_bytes;
    if (limit) *limit = d->cache_limit;
    if (entries) *entries = n;
    return PXQ_OK;
}

int pxq_matvec(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
               size_t ldy, const float* bias, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (int rc = check_matmul_args(w, row_first, row_count, input, columns, output, ldy)) return rc;
    return run_matmul(d, w, row_first, row_count, input, columns, output, ldy, bias, nullptr, 1,
                      static_cast<cudaStream_t>(stream));
}

int pxq_gemm(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
             size_t ldy, const float* bias, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (int rc = check_matmul_args(w, row_first, row_count, input, columns, output, ldy)) return rc;
    return run_matmul(d, w, row_first, row_count, input, columns, output, ldy, bias, nullptr, 2,
                      static_cast<cudaStream_t>(stream));
}

int pxq_matmul(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
               size_t ldy, const float* bias, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (int rc = check_matmul_args(w, row_first, row_count, input, columns, output, ldy)) return rc;
    return run_matmul(d, w, row_first, row_count, input, columns, output, ldy, bias, nullptr, 0,
                      static_cast<cudaStream_t>(stream));
}

int pxq_matmul_scatter(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns,
                       float* const* dsts, size_t ndst, size_t ldy, size_t col_offset, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!dsts || !ndst || ndst > (size_t)kMaxScatter) return fail(PXQ_ERR_INVALID, "1 to %d destinations (got %zu)", kMaxScatter, ndst);
    for (size_t k = 0; k < ndst; k++)
        if (!dsts[k]) return fail(PXQ_ERR_INVALID, "null destination %zu", k);
    if (int rc = check_matmul_args(w, row_first, row_count, input, columns, dsts[0], ldy)) return rc;
    if (columns <= 8) return fail(PXQ_ERR_UNSUPPORTED, "scatter runs on the GEMM path (more than 8 columns, got %zu)", columns);
    if (col_offset + row_count > ldy) return fail(PXQ_ERR_INVALID, "columns [%zu, %zu) outside ldy %zu", col_offset,
                                                  col_offset + row_count, ldy);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    pxq_activation* a = nullptr;
    int rc = quantize_activation(d, w->type, input, (int64_t)columns, w->inner, 2, &a, s);
    if (rc) return rc;
    // dsts[0]: this GPU's output, written like any output (TMA-store epilogue where aligned);
    // dsts[1..]: the peers', written from the same staged tiles
    rc = run_gemm(d, w, row_first, row_count, a, dsts[0] + col_offset, ldy, nullptr, nullptr, s, dsts + 1, (int)ndst - 1,
                  (int64_t)col_offset);
    free_activation(a, s);
    return rc;
}

int pxq_ipc_alloc(size_t bytes, void** ptr, void* handle)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!ptr || !handle || !bytes) return fail(PXQ_ERR_INVALID, "null pointer or zero bytes");
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_NO_MEMORY, "%zu bytes", bytes);
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return fail(PXQ_ERR_CUDA, "cudaIpcGetMemHandle failed");
    }
    static_assert(sizeof(h) == PXQ_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return PXQ_OK;
}

int pxq_ipc_free(void* ptr)
{
    if (ptr && cudaFree(ptr) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_CUDA, "cudaFree failed");
    }
    return PXQ_OK;
}

int pxq_ipc_open(const void* handle, void** ptr)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!handle || !ptr) return fail(PXQ_ERR_INVALID, "null handle or pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_CUDA, "cudaIpcOpenMemHandle failed");
    }
    *ptr = p;
    return PXQ_OK;
}

int pxq_ipc_close(void* ptr)
{
    if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_CUDA, "cudaIpcCloseMemHandle failed");
    }
    return PXQ_OK;
}

int pxq_matmul_gated(pxq_weight* w, const float* input, size_t columns, float* output, size_t ldy, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!w || !input || !output) return fail(PXQ_ERR_INVALID, "null weight, input or output");
    if (!w->gated) return fail(PXQ_ERR_INVALID, "weight was not uploaded with pxq_weight_upload_gated");
    if (!columns) return fail(PXQ_ERR_INVALID, "zero columns");
    const int64_t F = w->rows / 2;
    if (ldy < (size_t)F && columns > 1) return fail(PXQ_ERR_INVALID, "ldy %zu < %lld output rows", ldy, (long long)F);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (columns > 8) {
        // tensor-core GEMM over the interleaved 2F rows, silu(gate) * up in its epilogue
        pxq_activation* a = nullptr;
        int rc = quantize_activation(d, w->type, input, (int64_t)columns, w->inner, 2, &a, s);
        if (rc) return rc;
        rc = run_gemm(d, w, 0, (size_t)w->rows, a, output, ldy, nullptr, nullptr, s);
        free_activation(a, s);
        return rc;
    }
    if (w->type == kTypeQ5_K || w->type == kTypeQ6_K || w->inner % 256 == 0) {
        // one matvec: each CTA streams gate tile j and up tile j and writes silu(g) * u
        const MatvecPlan plan = plan_matvec(w->type, w->rows, w->inner, (int64_t)columns, d->sms, true, true);
        void* scratch = stream_scratch(t_device, s, plan.total_bytes);
        const bool own = scratch == nullptr;
        if (own && cudaMallocAsync(&scratch, plan.total_bytes, s) != cudaSuccess) {
            cudaGetLastError();
            return fail(PXQ_ERR_NO_MEMORY, "gated matvec scratch allocation of %zu bytes failed", plan.total_bytes);
        }
        cudaError_t e = matvec_fused(w, 0, (size_t)w->rows, input, output, ldy, nullptr, plan, static_cast<uint8_t*>(scratch),
                                     d->status, s);
        if (own) cudaFreeAsync(scratch, s);
        if (e != cudaSuccess) return fail(PXQ_ERR_CUDA, "gated matvec launch failed: %s", cudaGetErrorString(e));
        return PXQ_OK;
    }
    // Q8_0 with K not a multiple of 256: matvec over the 2F rows into scratch
    // after the matvec's own, then the epilogue
    const MatvecPlan plan = plan_matvec(w->type, w->rows, w->inner, (int64_t)columns, d->sms, true);
    const size_t off_s = (plan.total_bytes + 255) & ~(size_t)255;
    const size_t need = off_s + (size_t)columns * (size_t)w->rows * 4;
    void* scratch = stream_scratch(t_device, s, need);
    const bool own = scratch == nullptr;
    if (own && cudaMallocAsync(&scratch, need, s) != cudaSuccess) {
        cudaGetLastError();
        return fail(PXQ_ERR_NO_MEMORY, "gated matvec scratch allocation of %zu bytes failed", need);
    }
    if (own && plan.fused && plan.counter_bytes)  // fresh memory: no quantize kernel clears the counters
        PXQ_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(scratch) + plan.off_counters, 0, plan.counter_bytes, s));
    float* sums = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + off_s);
    cudaError_t e = matvec_fused(w, 0, (size_t)w->rows, input, sums, (size_t)w->rows, nullptr, plan,
                                 static_cast<uint8_t*>(scratch), d->status, s);
    if (e == cudaSuccess) e = counted(launch_gate_rows(sums, (int64_t)columns, F, output, (int64_t)ldy, s));
    if (own) cudaFreeAsync(scratch, s);
    if (e != cudaSuccess) return fail(PXQ_ERR_CUDA, "gated matvec launch failed: %s", cudaGetErrorString(e));
    return PXQ_OK;
}

int pxq_attention(const float* q, size_t q_rows, const float* k, const float* v, size_t k_rows, size_t heads,
                  size_t kv_heads, size_t head_dim, const pxq_attention_range* ranges, size_t nranges, size_t query_offset,
                  float* output, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    // the reference's argument checks (src/tensor.cpp:386-393)
    if (!q || !k || !v || !output) return fail(PXQ_ERR_INVALID, "null q, k, v or output");
    if (!heads || !kv_heads || heads % kv_heads || !q_rows || !k_rows) return fail(PXQ_ERR_INVALID, "bad head counts or sizes");
    if (heads > 0x7fffffffu || q_rows > 0x7fffffffu || k_rows > 0x7fffffffu) return fail(PXQ_ERR_UNSUPPORTED, "sizes exceed INT32_MAX");
    if (head_dim != 64 && head_dim != 80 && head_dim != 128)
        return fail(PXQ_ERR_UNSUPPORTED, "head size %zu (64, 80 and 128 are handled)", head_dim);
    int64_t ends[kAttnMaxRanges], keys[kAttnMaxRanges];
    int causal[kAttnMaxRanges];
    int n = 0;
    if (!ranges || !nranges) {
        ends[0] = (int64_t)q_rows;
        keys[0] = (int64_t)k_rows;
        causal[0] = 0;
        n = 1;
    } else {
        if (nranges > (size_t)kAttnMaxRanges) return fail(PXQ_ERR_UNSUPPORTED, "more than %d query ranges", kAttnMaxRanges);
        size_t covered = 0;
        for (size_t i = 0; i < nranges; i++) {
            const pxq_attention_range& r = ranges[i];
            if (r.query_begin != covered || r.query_end <= r.query_begin || r.query_end > q_rows || !r.key_end ||
                r.key_end > k_rows)
                return fail(PXQ_ERR_INVALID, "query range %zu does not continue [0, q_rows) or names keys outside [1, k_rows]", i);
            covered = r.query_end;
            ends[n] = (int64_t)r.query_end;
            keys[n] = (int64_t)r.key_end;
            causal[n] = r.causal ? 1 : 0;
            n++;
        }
        if (covered != q_rows) return fail(PXQ_ERR_INVALID, "query ranges cover %zu of %zu rows", covered, q_rows);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = attention_scratch_bytes((int64_t)q_rows, (int64_t)heads, (int64_t)kv_heads, (int64_t)head_dim, (int64_t)k_rows, d->sms);
    float* scratch = nullptr;
    if (need) {
        // past the matvec's counter region, which every call must leave zero
        uint8_t* base = static_cast<uint8_t*>(stream_scratch(t_device, s, kMvCounterRegion + need));
        if (!base) return fail(PXQ_ERR_NO_MEMORY, "attention scratch of %zu bytes", need);
        scratch = reinterpret_cast<float*>(base + kMvCounterRegion);
    }
    const cudaError_t e = launch_attention(q, (int64_t)q_rows, k, v, (int64_t)k_rows, (int)heads, (int)kv_heads, (int)head_dim,
                                           ends, keys, causal, n, (int64_t)query_offset, output, scratch, need, d->sms, s);
    if (counted(e, need ? 2 : 1) != cudaSuccess) return fail(PXQ_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    return PXQ_OK;
}

int pxq_gemm_block_dots(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* dump,
                        void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (int rc = check_matmul_args(w, row_first, row_count, input, columns, dump, row_count)) return rc;
    return run_matmul(d, w, row_first, row_count, input, columns, dump, row_count, nullptr, dump, 2,
                      static_cast<cudaStream_t>(stream));
}

int pxq_activation_quantize(uint32_t weight_type, const float* input, size_t columns, size_t inner, pxq_activation** out,
                            void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!out) return fail(PXQ_ERR_INVALID, "null out");
    return quantize_activation(d, weight_type, input, (int64_t)columns, (int64_t)inner, 0, out,
                               static_cast<cudaStream_t>(stream));
}

int pxq_matmul_quantized(pxq_weight* w, size_t row_first, size_t row_count, const pxq_activation* a, float* output,
                         size_t ldy, const float* bias, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (int rc = check_matmul_args(w, row_first, row_count, a, a ? (size_t)a->M : 0, output, ldy)) return rc;
    if (int rc = check_activation(w, a)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return a->blocks ? run_matvec(d, w, row_first, row_count, a, output, ldy, bias, s)
                     : run_gemm(d, w, row_first, row_count, a, output, ldy, bias, nullptr, s);
}

int pxq_activation_release(pxq_activation* a, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!a) return fail(PXQ_ERR_INVALID, "null activation");
    free_activation(a, static_cast<cudaStream_t>(stream));
    return PXQ_OK;
}

uint64_t pxq_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int pxq_synchronize(void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    PXQ_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    uint32_t st = 0;
    PXQ_CUDA(cudaMemcpy(&st, d->status, 4, cudaMemcpyDeviceToHost));
    if (st) {
        // A kernel gave up a bounded wait.  A matvec interrupted that way may
        // leave counts in the split-K counters of its scratch, which later
        // fused calls (no quantize kernel to clear them) rely on finding zero:
        // once the device is idle, zero every counter region on this device.
        cudaDeviceSynchronize();
        reset_scratch_counters(t_device);
        cudaMemset(d->status, 0, 4);
        return fail(PXQ_ERR_DEVICE_STATUS, "a kernel gave up waiting (status %u); scratch counters reset", st);
    }
    return PXQ_OK;
}

int pxq_debug_matvec_stall(pxq_weight* w, const float* input, size_t columns, float* output, int static_scratch, void* stream)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!w || !input || !output || w->gated) return fail(PXQ_ERR_INVALID, "null or gated weight, null input or output");
    if (w->type != kTypeQ5_K && w->type != kTypeQ6_K) return fail(PXQ_ERR_UNSUPPORTED, "K-quant weights only");
    if (!columns || columns > 8) return fail(PXQ_ERR_INVALID, "columns must be 1..8");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    MatvecPlan plan = plan_matvec(w->type, w->rows, w->inner, (int64_t)columns, d->sms, true);
    plan.debug_stall = true;
    void* scratch = static_scratch ? noalloc_scratch(t_device) : stream_scratch(t_device, s, plan.total_bytes);
    if (!scratch) return fail(PXQ_ERR_NO_MEMORY, "no scratch");
    if (static_scratch && plan.total_bytes > (size_t)PXQ_NOALLOC_SCRATCH_BYTES)
        return fail(PXQ_ERR_UNSUPPORTED, "the call does not fit the static scratch");
    cudaError_t e = matvec_fused(w, 0, (size_t)w->rows, input, output, (size_t)w->rows, nullptr, plan,
                                 static_cast<uint8_t*>(scratch), d->status, s);
    if (e != cudaSuccess) return fail(PXQ_ERR_CUDA, "matvec launch failed: %s", cudaGetErrorString(e));
    return PXQ_OK;
}

int pxq_gather_shards(const float* src, size_t shards, size_t columns, size_t shard_rows, float* dst, size_t ldy, void* stream)
{
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (!src || !dst || !shards || !columns || !shard_rows) return fail(PXQ_ERR_INVALID, "null pointer or zero size");
    if (ldy < shards * shard_rows) return fail(PXQ_ERR_INVALID, "ldy %zu < shards*shard_rows", ldy);
    PXQ_CUDA(counted(launch_gather_shards(src, shards, columns, shard_rows, dst, ldy, static_cast<cudaStream_t>(stream))));
    return PXQ_OK;
}

int pxq_matmul_host(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns, float* output,
                    size_t ldy)
{
    Pin pin_(w);
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    if (int rc = check_matmul_args(w, row_first, row_count, input, columns, output, ldy)) return rc;
    if (!t_stream || t_stream_device != t_device) {
        PXQ_CUDA(cudaStreamCreateWithFlags(&t_stream, cudaStreamNonBlocking));
        PXQ_CUDA(cudaStreamCreateWithFlags(&t_up, cudaStreamNonBlocking));
        PXQ_CUDA(cudaStreamCreateWithFlags(&t_down, cudaStreamNonBlocking));
        t_stream_device = t_device;
    }
    cudaStream_t s = t_stream;
    const size_t inner = (size_t)w->inner;
    const size_t out_elems = (columns - 1) * ldy + row_count;
    float* xin = nullptr;
    float* yout = nullptr;
    const size_t xbytes = columns * inner * sizeof(float), ybytes = out_elems * sizeof(float);
    if (cudaMallocAsync(&xin, xbytes, s) != cudaSuccess || cudaMallocAsync(&yout, ybytes, s) != cudaSuccess) {
        cudaGetLastError();
        if (xin) cudaFreeAsync(xin, s);
        return fail(PXQ_ERR_NO_MEMORY, "cannot allocate device buffers");
    }
    // Chunks of activation rows (GEMM path only): chunk i's upload, chunk
    // i-1's quantize + GEMM and chunk i-2's download run at the same time (the
    // link is full duplex).  Activation rows are quantized independently and
    // every output element depends on its own row only, so the result is the
    // same bit for bit as one call over all rows.
    // The first chunk is short (128 rows) and the next ones double up to the
    // full chunk size, so the downloads -- the longest stream of a large call
    // when the weight has more rows than its inner size -- start early and
    // do not wait for the next chunk's upload and GEMM.
    const size_t chunk = columns > 8 ? std::max<size_t>(512, (columns + 7) / 8) : columns;
    const size_t first = columns > 1024 ? 128 : chunk;
    int rc = PXQ_OK;
    cudaError_t e = cudaSuccess;
    cudaEvent_t ready = nullptr;  // buffers allocated on s (and the caller's output rows uploaded)
    e = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ready, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(t_up, ready, 0);
    // keep caller-owned output elements between rows (ldy > row_count) intact
    if (e == cudaSuccess && ldy != row_count && columns > 1) e = cudaMemcpyAsync(yout, output, ybytes, cudaMemcpyHostToDevice, t_up);
    std::vector<cudaEvent_t> evs;
    size_t c0 = 0, step = first;
    for (; c0 < columns && e == cudaSuccess && !rc; c0 += step, step = std::min(2 * step, chunk)) {
        const size_t cn = std::min(step, columns - c0);
        cudaEvent_t up = nullptr, done = nullptr;
        if ((e = cudaEventCreateWithFlags(&up, cudaEventDisableTiming)) != cudaSuccess) break;
        evs.push_back(up);
        if ((e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming)) != cudaSuccess) break;
        evs.push_back(done);
        e = cudaMemcpyAsync(xin + c0 * inner, input + c0 * inner, cn * inner * sizeof(float), cudaMemcpyHostToDevice, t_up);
        if (e == cudaSuccess) e = cudaEventRecord(up, t_up);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, up, 0);
        if (e != cudaSuccess) break;
        rc = run_matmul(d, w, row_first, row_count, xin + c0 * inner, cn, yout + c0 * ldy, ldy, nullptr, nullptr, 0, s);
        if (rc) break;
        e = cudaEventRecord(done, s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(t_down, done, 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(output + c0 * ldy, yout + c0 * ldy, ((cn - 1) * ldy + row_count) * sizeof(float),
                                cudaMemcpyDeviceToHost, t_down);
    }
    // the buffers are freed on s once every copy on the two copy streams is done
    cudaEvent_t fin_up = nullptr, fin_down = nullptr;
    if (cudaEventCreateWithFlags(&fin_up, cudaEventDisableTiming) == cudaSuccess) {
        cudaEventRecord(fin_up, t_up);
        cudaStreamWaitEvent(s, fin_up, 0);
    }
    if (cudaEventCreateWithFlags(&fin_down, cudaEventDisableTiming) == cudaSuccess) {
        cudaEventRecord(fin_down, t_down);
        cudaStreamWaitEvent(s, fin_down, 0);
    }
    cudaFreeAsync(xin, s);
    cudaFreeAsync(yout, s);
    const int sync_rc = pxq_synchronize(s);
    for (cudaEvent_t ev : evs) cudaEventDestroy(ev);
    if (ready) cudaEventDestroy(ready);
    if (fin_up) cudaEventDestroy(fin_up);
    if (fin_down) cudaEventDestroy(fin_down);
    if (e != cudaSuccess) return fail(PXQ_ERR_CUDA, "copy failed: %s", cudaGetErrorString(e));
    if (rc) return rc;
    return sync_rc;
}

int pxq_quant_matmul(const unsigned char* weights, uint32_t type, const float* input, float* output, size_t rows,
                     size_t columns, size_t inner)
{
    // the reference's "not handled" cases (src/kernels_quant.cpp:373-377)
    if (type != PXQ_TYPE_Q8_0 && type != PXQ_TYPE_Q5_K && type != PXQ_TYPE_Q6_K)
        return fail(PXQ_ERR_UNSUPPORTED, "type %u not handled", type);
    const size_t block = type == PXQ_TYPE_Q8_0 ? 32 : 256;
    if (!rows || !columns || !inner || inner % block || inner > 0x7fffffffu)
        return fail(PXQ_ERR_UNSUPPORTED, "shape rows=%zu columns=%zu inner=%zu not handled", rows, columns, inner);
    if (!weights || !input || !output) return fail(PXQ_ERR_INVALID, "null pointer");
    DeviceCtx* d;
    if (int rc = ensure_device(&d)) return rc;
    // The device copy is cached under the host address, the shape and a
    // fingerprint of the bytes: a weight freed and replaced at the same
    // address gets its own entry (and the stale one is dropped) instead of
    // the old device copy.
    const uint64_t nbytes = pxq_weight_bytes(inner, rows, type);
    const uint64_t fp = fingerprint(weights, nbytes);
    char prefix[96], key[128];
    snprintf(prefix, sizeof(prefix), "host:%p:%zu:%zu:%u:", (const void*)weights, rows, inner, type);
    snprintf(key, sizeof(key), "%s%016llx", prefix, (unsigned long long)fp);
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        std::vector<pxq_weight*> stale;
        for (auto& kv : g_cache)
            if (kv.second->internal && !kv.second->pins && kv.first.compare(0, strlen(prefix), prefix) == 0 && kv.first != key)
                stale.push_back(kv.second);
        if (!stale.empty()) {
            cudaDeviceSynchronize();
            for (pxq_weight* w : stale) {
                uncache(w);
                delete w;
            }
        }
    }
    pxq_weight* w = nullptr;
    if (int rc = pxq_weight_upload(weights, 0, type, inner, rows, key, &w)) return rc;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        w->internal = true;
    }
    return pxq_matmul_host(w, 0, rows, input, columns, output, rows);
}

}  // extern "C"
