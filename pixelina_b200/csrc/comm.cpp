// comm.cpp -- the N-sharded multi-GPU matmul behind the C ABI (one process
// per GPU, NCCL over NVLink / NVSwitch).
//
// Every output column n of cpu_quant_matmul (one weight row) is independent
// of the others (src/kernels_quant.cpp:390-398), so the weight rows split
// evenly over G ranks: rank r holds rows [r*N/G, (r+1)*N/G) as an ordinary
// pxq_weight and computes Y[:, its columns] for all activation rows; every
// rank quantizes the replicated activation itself (identical bytes), so the
// assembled Y is bit-identical to a one-GPU run.  Two ways to assemble Y on
// every rank:
//   * fused (pxq_sharded_output): each rank's GEMM epilogue stores its
//     columns straight into every rank's output buffer (CUDA IPC mappings,
//     plain stores over NVLink) while later tiles compute, between two
//     device-side barriers (one-element NCCL all-reduces): before, every
//     rank is done with the buffer's previous contents; after, every
//     rank's stores have landed;
//   * all-gather: local GEMM into [M][N/G] scratch, ncclAllGather to
//     [G][M][N/G], one re-layout kernel (pxq_gather_shards) into [M][ldy].
//
// Failure handling: the communicator is created non-blocking and every
// wait polls ncclCommGetAsyncError and the stream against a host-side
// deadline; on expiry the communicator is aborted (in-flight NCCL kernels
// exit) and the call returns PXQ_ERR_TIMEOUT.  A rank that never joins, or
// never reaches a collective, therefore surfaces as an error on the others
// instead of a hang.  This file uses only the public C ABI of libpxq for
// the compute (pxq_matmul_scatter, pxq_matmul, pxq_gather_shards, IPC).
//
// NCCL is bound at the first communicator call (dlopen of libnccl.so.2, or
// PXQ_NCCL_LIBRARY), not linked: a process that never uses the multi-GPU
// path loads no NCCL, and one that has loaded an NCCL already (PyTorch's
// own) keeps using that one.
#include <dlfcn.h>

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>

#include <cuda_runtime.h>
#include <nccl.h>

#include "pxq.h"

namespace pxq {
void record_error(const char* msg);
}

namespace {

int comm_fail(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    pxq::record_error(buf);
    return code;
}

constexpr int kMaxRanks = 8;  // one node: the scatter writes at most 8 destinations

// The NCCL entry points this file uses, resolved from the loaded library.
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string error;
};

const NcclApi& nccl()
{
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* path = getenv("PXQ_NCCL_LIBRARY");
        void* h = nullptr;
        if (path && *path) {
            h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
        } else {
            h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);  // already in the process
            if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        }
        if (!h) {
            const char* e = dlerror();
            api.error = std::string("cannot load NCCL: ") + (e ? e : "libnccl.so.2 not found");
            return;
        }
        bool all = true;
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) {
                all = false;
                api.error = std::string("NCCL lacks ") + name;
            }
        };
        sym(api.GetUniqueId, "ncclGetUniqueId");
        sym(api.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(api.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(api.CommAbort, "ncclCommAbort");
        sym(api.CommFinalize, "ncclCommFinalize");
        sym(api.CommDestroy, "ncclCommDestroy");
        sym(api.AllReduce, "ncclAllReduce");
        sym(api.AllGather, "ncclAllGather");
        sym(api.GetErrorString, "ncclGetErrorString");
        api.ok = all;
    });
    return api;
}

const char* nccl_error(ncclResult_t r) { return nccl().GetErrorString ? nccl().GetErrorString(r) : "?"; }

}  // namespace

struct pxq_comm {
    ncclComm_t nccl = nullptr;
    int world = 0, rank = 0, device = 0;
    int timeout_ms = 0;
    bool broken = false;         // aborted after a timeout or an NCCL error: every later call fails
    int* flag = nullptr;         // device word reduced by the barriers
    cudaStream_t stream = nullptr;  // host-buffer calls
    // host-buffer calls: device copies of the input and a cached fused output
    float* xin = nullptr;
    size_t xin_bytes = 0;
    pxq_sharded_out* hout = nullptr;
};

struct pxq_sharded_out {
    pxq_comm* comm = nullptr;
    size_t columns = 0, ldy = 0;
    float* local = nullptr;             // this rank's buffer
    float* dsts[kMaxRanks] = {};        // this rank's buffer, then every other rank's (mapped)
    int ndst = 0;
};

namespace {

using clk = std::chrono::steady_clock;

// Abort the communicator after a failure; in-flight NCCL kernels exit.
void comm_break(pxq_comm* c)
{
    if (c->nccl) nccl().CommAbort(c->nccl);
    c->nccl = nullptr;
    c->broken = true;
}

// Wait until `s` has drained (or, with s == nullptr, until the communicator
// is ready), polling NCCL's asynchronous error state against the deadline.
int comm_wait(pxq_comm* c, cudaStream_t s, const char* what)
{
    const auto deadline = clk::now() + std::chrono::milliseconds(c->timeout_ms);
    while (true) {
        ncclResult_t ar = ncclSuccess;
        if (nccl().CommGetAsyncError(c->nccl, &ar) != ncclSuccess) ar = ncclInternalError;
        if (ar != ncclSuccess && ar != ncclInProgress) {
            comm_break(c);
            return comm_fail(PXQ_ERR_CUDA, "%s: NCCL error %d (%s); communicator aborted", what, (int)ar, nccl_error(ar));
        }
        bool done;
        if (s == nullptr) {
            done = ar == ncclSuccess;
        } else {
            const cudaError_t q = cudaStreamQuery(s);
            if (q != cudaSuccess && q != cudaErrorNotReady) {
                comm_break(c);
                return comm_fail(PXQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(q));
            }
            done = q == cudaSuccess && ar == ncclSuccess;
        }
        if (done) return PXQ_OK;
        if (clk::now() > deadline) {
            comm_break(c);
            return comm_fail(PXQ_ERR_TIMEOUT, "%s: not complete after %d ms (a rank missing?); communicator aborted", what,
                             c->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// A non-blocking NCCL call: ncclInProgress is a normal return.
bool nccl_ok(ncclResult_t r) { return r == ncclSuccess || r == ncclInProgress; }

// After a call on a non-blocking communicator returned ncclInProgress (a
// collective whose connections NCCL is still setting up in the background,
// typically the first of its kind), NCCL takes no further call on the
// communicator until its state is ncclSuccess again: poll it, against the
// deadline.  This waits for the call to be queued, not for its completion on
// the device.  On an error or a timeout the communicator is aborted.
int nccl_queued(pxq_comm* c, ncclResult_t r, const char* what)
{
    if (r == ncclSuccess) return PXQ_OK;
    if (r != ncclInProgress) {
        comm_break(c);
        return comm_fail(PXQ_ERR_CUDA, "%s could not be queued: NCCL error %d (%s); communicator aborted", what, (int)r,
                         nccl_error(r));
    }
    const auto deadline = clk::now() + std::chrono::milliseconds(c->timeout_ms);
    while (true) {
        ncclResult_t ar = ncclSuccess;
        if (nccl().CommGetAsyncError(c->nccl, &ar) != ncclSuccess) ar = ncclInternalError;
        if (ar == ncclSuccess) return PXQ_OK;
        if (ar != ncclInProgress) {
            comm_break(c);
            return comm_fail(PXQ_ERR_CUDA, "%s: NCCL error %d (%s); communicator aborted", what, (int)ar, nccl_error(ar));
        }
        if (clk::now() > deadline) {
            comm_break(c);
            return comm_fail(PXQ_ERR_TIMEOUT, "%s: not queued after %d ms (a rank missing?); communicator aborted", what,
                             c->timeout_ms);
        }
        std::this_thread::yield();
    }
}

int check_comm(pxq_comm* c)
{
    if (!c) return comm_fail(PXQ_ERR_INVALID, "null communicator");
    if (c->broken || !c->nccl) return comm_fail(PXQ_ERR_INVALID, "communicator was aborted after an earlier failure");
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != c->device) {
        if (cudaSetDevice(c->device) != cudaSuccess) return comm_fail(PXQ_ERR_CUDA, "cannot select device %d", c->device);
    }
    return PXQ_OK;
}

// Device-ordered barrier of all ranks on `s`.
int comm_barrier(pxq_comm* c, cudaStream_t s)
{
    return nccl_queued(c, nccl().AllReduce(c->flag, c->flag, 1, ncclInt32, ncclMax, c->nccl, s), "barrier all-reduce");
}

}  // namespace

extern "C" {

int pxq_comm_unique_id(void* id)
{
    if (!id) return comm_fail(PXQ_ERR_INVALID, "null id");
    static_assert(sizeof(ncclUniqueId) == PXQ_COMM_ID_BYTES, "id size");
    if (!nccl().ok) return comm_fail(PXQ_ERR_UNSUPPORTED, "%s", nccl().error.c_str());
    ncclUniqueId u;
    const ncclResult_t r = nccl().GetUniqueId(&u);
    if (r != ncclSuccess) return comm_fail(PXQ_ERR_CUDA, "ncclGetUniqueId failed: %s", nccl_error(r));
    std::memcpy(id, &u, sizeof(u));
    return PXQ_OK;
}

int pxq_comm_init(const void* id, int world, int rank, int timeout_ms, pxq_comm** out)
{
    if (!id || !out) return comm_fail(PXQ_ERR_INVALID, "null id or out");
    *out = nullptr;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return comm_fail(PXQ_ERR_INVALID, "rank %d of world %d (1..%d ranks)", rank, world, kMaxRanks);
    if (timeout_ms <= 0) return comm_fail(PXQ_ERR_INVALID, "timeout_ms must be positive");
    if (!nccl().ok) return comm_fail(PXQ_ERR_UNSUPPORTED, "%s", nccl().error.c_str());
    // the calling thread's device (pxq_init selects it)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return comm_fail(PXQ_ERR_NO_DEVICE, "no current CUDA device");
    auto* c = new pxq_comm();
    c->world = world;
    c->rank = rank;
    c->device = dev;
    c->timeout_ms = timeout_ms;
    if (cudaMalloc(&c->flag, 256) != cudaSuccess || cudaMemset(c->flag, 0, 256) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        if (c->flag) cudaFree(c->flag);
        delete c;
        return comm_fail(PXQ_ERR_NO_MEMORY, "cannot allocate the communicator's device state");
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = nccl().CommInitRankConfig(&c->nccl, world, u, rank, &cfg);
    if (!nccl_ok(r)) {
        if (c->nccl) nccl().CommAbort(c->nccl);
        cudaFree(c->flag);
        cudaStreamDestroy(c->stream);
        delete c;
        return comm_fail(PXQ_ERR_CUDA, "ncclCommInitRankConfig failed: %s", nccl_error(r));
    }
    if (int rc = comm_wait(c, nullptr, "communicator set-up")) {
        cudaFree(c->flag);
        cudaStreamDestroy(c->stream);
        delete c;
        return rc;
    }
    *out = c;
    return PXQ_OK;
}

int pxq_comm_size(const pxq_comm* comm, int* world, int* rank)
{
    if (!comm) return comm_fail(PXQ_ERR_INVALID, "null communicator");
    if (world) *world = comm->world;
    if (rank) *rank = comm->rank;
    return PXQ_OK;
}

int pxq_comm_barrier(pxq_comm* comm)
{
    if (int rc = check_comm(comm)) return rc;
    if (int rc = comm_barrier(comm, comm->stream)) return rc;
    return comm_wait(comm, comm->stream, "barrier");
}

int pxq_comm_synchronize(pxq_comm* comm, void* stream)
{
    if (int rc = check_comm(comm)) return rc;
    if (int rc = comm_wait(comm, static_cast<cudaStream_t>(stream), "stream synchronize")) return rc;
    return pxq_synchronize(stream);
}

int pxq_comm_destroy(pxq_comm* comm)
{
    if (!comm) return comm_fail(PXQ_ERR_INVALID, "null communicator");
    if (comm->hout) pxq_sharded_output_destroy(comm->hout);
    if (comm->nccl) {
        cudaStreamSynchronize(comm->stream);
        // finalize (flushes outstanding work) with a deadline, then destroy
        if (nccl_ok(nccl().CommFinalize(comm->nccl)) && comm_wait(comm, nullptr, "communicator finalize") == PXQ_OK)
            nccl().CommDestroy(comm->nccl);
        comm->nccl = nullptr;
    }
    if (comm->xin) cudaFree(comm->xin);
    if (comm->flag) cudaFree(comm->flag);
    if (comm->stream) cudaStreamDestroy(comm->stream);
    delete comm;
    return PXQ_OK;
}

int pxq_sharded_output_create(pxq_comm* comm, size_t columns, size_t ldy, pxq_sharded_out** out, float** local)
{
    if (int rc = check_comm(comm)) return rc;
    if (!out || !columns || !ldy) return comm_fail(PXQ_ERR_INVALID, "null out or zero size");
    *out = nullptr;
    auto* o = new pxq_sharded_out();
    o->comm = comm;
    o->columns = columns;
    o->ldy = ldy;
    const int G = comm->world;
    // this rank's buffer and its IPC handle; every rank's handle through one all-gather
    unsigned char handle[PXQ_IPC_HANDLE_BYTES];
    void* buf = nullptr;
    if (int rc = pxq_ipc_alloc(columns * ldy * sizeof(float), &buf, handle)) {
        delete o;
        return rc;
    }
    o->local = static_cast<float*>(buf);
    unsigned char* dh = nullptr;
    unsigned char all[kMaxRanks * PXQ_IPC_HANDLE_BYTES];
    int rc = PXQ_OK;
    if (cudaMalloc(&dh, (size_t)G * PXQ_IPC_HANDLE_BYTES) != cudaSuccess) {
        cudaGetLastError();
        rc = comm_fail(PXQ_ERR_NO_MEMORY, "handle exchange buffer");
    }
    if (!rc && cudaMemcpyAsync(dh + (size_t)comm->rank * PXQ_IPC_HANDLE_BYTES, handle, PXQ_IPC_HANDLE_BYTES,
                               cudaMemcpyHostToDevice, comm->stream) != cudaSuccess)
        rc = comm_fail(PXQ_ERR_CUDA, "handle upload failed");
    if (!rc)
        rc = nccl_queued(comm,
                         nccl().AllGather(dh + (size_t)comm->rank * PXQ_IPC_HANDLE_BYTES, dh, PXQ_IPC_HANDLE_BYTES, ncclUint8,
                                          comm->nccl, comm->stream),
                         "handle all-gather");
    if (!rc) rc = comm_wait(comm, comm->stream, "output handle exchange");
    if (!rc && cudaMemcpy(all, dh, (size_t)G * PXQ_IPC_HANDLE_BYTES, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = comm_fail(PXQ_ERR_CUDA, "handle download failed");
    if (dh) cudaFree(dh);
    o->dsts[0] = o->local;
    o->ndst = 1;
    for (int r = 0; r < G && !rc; r++) {
        if (r == comm->rank) continue;
        void* p = nullptr;
        rc = pxq_ipc_open(all + (size_t)r * PXQ_IPC_HANDLE_BYTES, &p);
        if (!rc) o->dsts[o->ndst++] = static_cast<float*>(p);
    }
    if (rc) {
        for (int k = 1; k < o->ndst; k++) pxq_ipc_close(o->dsts[k]);
        pxq_ipc_free(o->local);
        delete o;
        return rc;
    }
    *out = o;
    if (local) *local = o->local;
    return PXQ_OK;
}

int pxq_sharded_output_destroy(pxq_sharded_out* o)
{
    if (!o) return comm_fail(PXQ_ERR_INVALID, "null output");
    pxq_comm* c = o->comm;
    cudaDeviceSynchronize();
    for (int k = 1; k < o->ndst; k++) pxq_ipc_close(o->dsts[k]);
    int rc = PXQ_OK;
    // every rank has closed its mapping of this buffer before it is freed
    if (c && c->nccl && !c->broken) rc = pxq_comm_barrier(c);
    pxq_ipc_free(o->local);
    if (c && c->hout == o) c->hout = nullptr;
    delete o;
    return rc;
}

int pxq_sharded_matmul(pxq_comm* comm, pxq_weight* shard, size_t shard_rows, const float* input, size_t columns,
                       pxq_sharded_out* out, float* output, size_t ldy, void* stream)
{
    if (int rc = check_comm(comm)) return rc;
    if (!shard || !input || !columns || !shard_rows) return comm_fail(PXQ_ERR_INVALID, "null shard or input, or zero size");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int G = comm->world;
    const size_t rows = shard_rows * (size_t)G;
    const size_t col_off = shard_rows * (size_t)comm->rank;
    if (out) {
        // fused: the GEMM stores into every rank's buffer
        if (out->comm != comm) return comm_fail(PXQ_ERR_INVALID, "output belongs to another communicator");
        if (out->columns != columns || out->ldy < rows)
            return comm_fail(PXQ_ERR_INVALID, "output is [%zu][%zu], the call needs [%zu][>= %zu]", out->columns, out->ldy, columns,
                             rows);
        if (columns <= 8) {
            // the scatter runs on the GEMM path; a few columns go through the
            // matvec into the local buffer and an all-gather of the same layout
            return comm_fail(PXQ_ERR_UNSUPPORTED, "the fused sharded path needs more than 8 activation rows (got %zu)", columns);
        }
        if (int rc = comm_barrier(comm, s)) return rc;  // every rank is done with its buffer's previous contents
        if (int rc = pxq_matmul_scatter(shard, 0, shard_rows, input, columns, out->dsts, (size_t)out->ndst, out->ldy, col_off, s))
            return rc;
        return comm_barrier(comm, s);  // every rank's stores have landed
    }
    // all-gather: local shard, NCCL all-gather, re-layout
    if (!output || ldy < rows) return comm_fail(PXQ_ERR_INVALID, "null output or ldy %zu < %zu", ldy, rows);
    float* local = nullptr;
    float* gathered = nullptr;
    const size_t block = columns * shard_rows;
    if (cudaMallocAsync(&local, block * sizeof(float), s) != cudaSuccess ||
        cudaMallocAsync(&gathered, block * (size_t)G * sizeof(float), s) != cudaSuccess) {
        cudaGetLastError();
        if (local) cudaFreeAsync(local, s);
        return comm_fail(PXQ_ERR_NO_MEMORY, "all-gather scratch of %zu bytes", block * (size_t)(G + 1) * sizeof(float));
    }
    int rc = pxq_matmul(shard, 0, shard_rows, input, columns, local, shard_rows, nullptr, s);
    if (!rc) rc = nccl_queued(comm, nccl().AllGather(local, gathered, block, ncclFloat32, comm->nccl, s), "all-gather");
    if (!rc) rc = pxq_gather_shards(gathered, (size_t)G, columns, shard_rows, output, ldy, s);
    cudaFreeAsync(local, s);
    cudaFreeAsync(gathered, s);
    return rc;
}

int pxq_sharded_matmul_host(pxq_comm* comm, pxq_weight* shard, size_t shard_rows, const float* input, size_t columns,
                            size_t inner, float* output)
{
    if (int rc = check_comm(comm)) return rc;
    if (!shard || !input || !output || !columns || !inner || !shard_rows)
        return comm_fail(PXQ_ERR_INVALID, "null pointer or zero size");
    const size_t rows = shard_rows * (size_t)comm->world;
    cudaStream_t s = comm->stream;
    const size_t xbytes = columns * inner * sizeof(float);
    if (comm->xin_bytes < xbytes) {
        if (comm->xin) cudaFree(comm->xin);
        comm->xin = nullptr;
        comm->xin_bytes = 0;
        if (cudaMalloc(&comm->xin, xbytes) != cudaSuccess) {
            cudaGetLastError();
            return comm_fail(PXQ_ERR_NO_MEMORY, "input buffer of %zu bytes", xbytes);
        }
        comm->xin_bytes = xbytes;
    }
    // the output buffers are created collectively on first use (every rank
    // makes the same calls) and kept for calls of the same shape
    if (comm->hout && (comm->hout->columns != columns || comm->hout->ldy != rows)) {
        if (int rc = pxq_sharded_output_destroy(comm->hout)) return rc;
    }
    if (!comm->hout) {
        pxq_sharded_out* o = nullptr;
        if (int rc = pxq_sharded_output_create(comm, columns, rows, &o, nullptr)) return rc;
        comm->hout = o;
    }
    if (cudaMemcpyAsync(comm->xin, input, xbytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return comm_fail(PXQ_ERR_CUDA, "input upload failed");
    if (int rc = pxq_sharded_matmul(comm, shard, shard_rows, comm->xin, columns, comm->hout, nullptr, 0, s)) return rc;
    if (cudaMemcpyAsync(output, comm->hout->local, columns * rows * sizeof(float), cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return comm_fail(PXQ_ERR_CUDA, "output download failed");
    return pxq_comm_synchronize(comm, s);
}

}  // extern "C"
