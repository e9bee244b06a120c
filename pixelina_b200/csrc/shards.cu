// shards.cu -- output re-layout for the N-sharded multi-GPU matmul.
//
// Each rank computes Y[:, shard] into a dense [columns][shard_rows] block;
// an all-gather of those blocks yields [shards][columns][shard_rows].  The
// consumer wants row-major [columns][N]; this kernel performs that one copy
// with 16-byte accesses when the shapes allow it.
#include "pxq_internal.h"

namespace pxq {
namespace {

__global__ void k_gather_shards(const float* __restrict__ src, int64_t shards, int64_t columns, int64_t shard_rows,
                                float* __restrict__ dst, int64_t ldy)
{
    const int64_t total = shards * columns * shard_rows;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i % shard_rows;
        const int64_t c = (i / shard_rows) % columns;
        const int64_t s = i / (shard_rows * columns);
        dst[c * ldy + s * shard_rows + r] = src[i];
    }
}

__global__ void k_gather_shards4(const float4* __restrict__ src, int64_t shards, int64_t columns, int64_t shard_rows4,
                                 float* __restrict__ dst, int64_t ldy)
{
    const int64_t total = shards * columns * shard_rows4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r4 = i % shard_rows4;
        const int64_t c = (i / shard_rows4) % columns;
        const int64_t s = i / (shard_rows4 * columns);
        *reinterpret_cast<float4*>(dst + c * ldy + (s * shard_rows4 + r4) * 4) = src[i];
    }
}

}  // namespace

cudaError_t launch_gather_shards(const float* src, int64_t shards, int64_t columns, int64_t shard_rows, float* dst,
                                 int64_t ldy, cudaStream_t s)
{
    const int threads = 256;
    const bool vec = (shard_rows % 4 == 0) && (ldy % 4 == 0) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) &&
                     ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
    const int64_t work = vec ? shards * columns * shard_rows / 4 : shards * columns * shard_rows;
    int64_t blocks = (work + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    if (vec)
        k_gather_shards4<<<(int)blocks, threads, 0, s>>>(reinterpret_cast<const float4*>(src), shards, columns, shard_rows / 4,
                                                        dst, ldy);
    else
        k_gather_shards<<<(int)blocks, threads, 0, s>>>(src, shards, columns, shard_rows, dst, ldy);
    return cudaGetLastError();
}

}  // namespace pxq
