// noalloc.cu -- the decode matvec with no device allocation per call.
//
// Who needs this: callers that cannot call cudaMalloc (or any allocating
// routine) at the point where they multiply -- a decode loop that must not
// stall on the allocator, code running inside a region where the caller has
// forbidden allocation, or an embedding application whose device-memory
// budget is fixed up front.  pxq_matvec quantizes the activation rows into
// stream-ordered scratch from the CUDA memory pool; this variant quantizes
// them into one fixed array that lives in this library's device data instead,
// so a successful call only launches two kernels (quantize, matvec) and makes
// no device allocation.  (A rejected call records its message for
// pxq_last_error() in host memory.)
//
// The array: g_noalloc_scratch, PXQ_NOALLOC_SCRATCH_BYTES (4 MiB) per device
// that loads the library, held until the process exits.  Host code never
// touches it by name (its host-side symbol is not a device address): on the
// first call on each device, with that device current, the address is looked
// up once with cudaGetSymbolAddress and cached.  That first call therefore
// does the set-up (and may make the runtime load this module); make it before
// any stream capture.
//
// Layout of the array per call: the matvec's counters (a region of their
// own), the quantized activation rows (none when the matvec quantizes a small
// activation itself), then its fp32 partial sums.  The counters must start
// at zero: the array starts zeroed, the quantize kernel of a call (when there
// is one) clears them, every completed matvec leaves them zero, and after a
// call whose bounded wait ran out (pxq_synchronize reports
// PXQ_ERR_DEVICE_STATUS) pxq_synchronize clears them again; every other byte
// the kernels read is written earlier in the same call.
//
// Sharing: every call on a device uses the same array and it keeps the last
// call's contents.  Two calls whose work overlaps on the GPU (different
// streams without ordering) race on the array; order them on one stream or
// with events.
#include <cstdio>
#include <mutex>

#include "pxq.h"
#include "pxq_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[PXQ_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 16;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

// Helpers defined in api.cu: read-only view of a weight handle, and the
// message returned by pxq_last_error().
namespace pxq {
bool weight_view(const pxq_weight* w, uint32_t* type, int64_t* inner, int64_t* rows, int64_t* stride, const uint8_t** raw,
                 int* device);
void record_error(const char* msg);
int device_sm_count(int device);
uint32_t* device_status(int device);
cudaError_t matvec_fused(const pxq_weight* w, size_t row_first, size_t row_count, const float* input, float* output,
                         size_t ldy, const float* bias, const MatvecPlan& plan, uint8_t* scratch, uint32_t* status,
                         cudaStream_t s);
}

namespace {
int noalloc_fail(int code, const char* msg)
{
    pxq::record_error(msg);
    return code;
}
}  // namespace

namespace pxq {
// The array's device address on `device` (with that device current): looked
// up once per device with cudaGetSymbolAddress -- the host-side symbol is not
// a device address -- and cached.  Null if the look-up fails.
void* noalloc_scratch(int device)
{
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return nullptr;
        }
        g_scratch_ptr[device] = p;
    }
    return g_scratch_ptr[device];
}

// Zero the counter region (after a call that a bounded wait interrupted may
// have left counts in it; the caller has synchronized the device).  No-op
// when the array was never set up on `device`.
cudaError_t noalloc_clear_counters(int device)
{
    void* p = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (device >= 0 && device < kMaxDevices) p = g_scratch_ptr[device];
    }
    return p ? cudaMemset(p, 0, kMvCounterRegion) : cudaSuccess;
}
}  // namespace pxq

extern "C" int pxq_matvec_noalloc(pxq_weight* w, size_t row_first, size_t row_count, const float* input, size_t columns,
                                  float* output, size_t ldy, const float* bias, void* stream)
{
    uint32_t type = 0;
    int64_t inner = 0, rows = 0, stride = 0;
    const uint8_t* raw = nullptr;
    int wdev = -1;
    if (!w || !input || !output || !pxq::weight_view(w, &type, &inner, &rows, &stride, &raw, &wdev))
        return noalloc_fail(PXQ_ERR_INVALID, "null or gated weight, null input or output");
    if (!columns || !row_count || columns > 8)
        return noalloc_fail(PXQ_ERR_INVALID, "columns must be 1..8 and row_count > 0");
    if (row_first > (size_t)rows || row_count > (size_t)rows - row_first)
        return noalloc_fail(PXQ_ERR_INVALID, "row range outside the weight");
    if (ldy < row_count && columns > 1) return noalloc_fail(PXQ_ERR_INVALID, "ldy < row_count");
    if (type != pxq::kTypeQ8_0 && type != pxq::kTypeQ5_K && type != pxq::kTypeQ6_K)
        return noalloc_fail(PXQ_ERR_UNSUPPORTED, "weight type not supported");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return noalloc_fail(PXQ_ERR_NO_DEVICE, "no current CUDA device");
    if (dev != wdev) return noalloc_fail(PXQ_ERR_INVALID, "the weight lives on another device than the current one");
    // the static array holds the quantized activation rows and the matvec's
    // partial sums and counters
    const pxq::MatvecPlan plan = pxq::plan_matvec(type, (int64_t)row_count, inner, (int64_t)columns, pxq::device_sm_count(dev),
                                                  true);
    const uint64_t need = plan.total_bytes;
    if (need > PXQ_NOALLOC_SCRATCH_BYTES) {
        char msg[200];
        snprintf(msg, sizeof(msg), "this call needs %llu bytes of scratch; the static scratch holds %d bytes "
                 "(PXQ_NOALLOC_SCRATCH_BYTES)", (unsigned long long)need, PXQ_NOALLOC_SCRATCH_BYTES);
        return noalloc_fail(PXQ_ERR_UNSUPPORTED, msg);
    }
    void* scratch = pxq::noalloc_scratch(dev);
    if (!scratch) return noalloc_fail(PXQ_ERR_CUDA, "cudaGetSymbolAddress of the static scratch failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = pxq::matvec_fused(w, row_first, row_count, input, output, ldy, bias, plan,
                                            static_cast<uint8_t*>(scratch), pxq::device_status(dev), s);
    if (e != cudaSuccess) {
        char msg[200];
        snprintf(msg, sizeof(msg), "kernel launch failed: %s", cudaGetErrorString(e));
        return noalloc_fail(PXQ_ERR_CUDA, msg);
    }
    return PXQ_OK;
}
