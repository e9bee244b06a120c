// epilogue.cu -- the gated feed-forward epilogue for the matvec path.
//
// A gated weight holds a feed-forward's gate projection (F rows) and up
// projection (F rows); the matvec computes both into s[c][2F], and this kernel
// finishes the callers' tensor_silu + tensor_gate (src/tensor.cpp:199-208,
// :334-345; called at src/inference.cpp:331-334, src/qwen_vl.cpp:396-399,
// src/qwen_image.cpp:271-274):  y[c][n] = (g / (1 + exp(-g))) * u  with
// g = s[c][n], u = s[c][F + n], the same operation order in fp32.
#include "pxq_device.cuh"
#include "pxq_internal.h"

namespace pxq {
namespace {

__global__ void k_gate_rows(const float* __restrict__ s, int64_t columns, int64_t F, float* __restrict__ y, int64_t ldy)
{
    griddep_wait();  // s is written by the preceding matvec
    const int64_t total = columns * F;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i / F, n = i % F;
        const float g = s[c * 2 * F + n], u = s[c * 2 * F + F + n];
        y[c * ldy + n] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
}

}  // namespace

cudaError_t launch_gate_rows(const float* s, int64_t columns, int64_t F, float* y, int64_t ldy, cudaStream_t st)
{
    int64_t blocks = (columns * F + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    return launch_pdl(k_gate_rows, dim3((unsigned)blocks), dim3(256), 0, st, s, columns, F, y, ldy);
}

}  // namespace pxq
