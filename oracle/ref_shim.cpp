/*
 * ref_shim.cpp -- C entry points into Pixelina's own CPU kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
 * with the reference's unmodified sources, read in place from the Pixelina
 * tree (REF=... on the make command line), into oracle/_ref/libpixref.so.
 * It is used to pin the C restatement in pxq_oracle.c and, in bench.py's
 * reference arm, as the timed CPU baseline.  Nothing here is shipped.
 *
 * The quantize and dot helpers of the reference are file-static, so the
 * reference translation unit src/kernels_quant.cpp is included here whole
 * (unmodified) to reach them; everything else links against the reference's
 * other objects (tensor.cpp for cpu_parallel, backend_cpu.cpp for cpu_decode,
 * model.cpp for weight_bytes, ...).
 */
#include "kernels_quant.cpp"

extern "C" {

void pixref_quantize_q8_0(const float* x, void* y, int64_t k)
{
    quantize_row_q8_0_ref(x, static_cast<block_q8_0*>(y), k);
}

void pixref_quantize_q8_K(const float* x, void* y, int64_t k)
{
    quantize_row_q8_K_ref(x, static_cast<block_q8_K*>(y), k);
}

float pixref_dot_q8_0(int n, const void* x, const void* y)
{
    return pix_dot_q8_0(n, static_cast<const block_q8_0*>(x), static_cast<const block_q8_0*>(y));
}

float pixref_dot_q5_K(int n, const void* x, const void* y)
{
    return pix_dot_q5_K(n, static_cast<const block_q5_K*>(x), static_cast<const block_q8_K*>(y));
}

float pixref_dot_q6_K(int n, const void* x, const void* y)
{
    return pix_dot_q6_K(n, static_cast<const block_q6_K*>(x), static_cast<const block_q8_K*>(y));
}

int pixref_quant_matmul(const unsigned char* weights, uint32_t type, const float* input, float* output, size_t rows, size_t columns, size_t inner)
{
    return cpu_quant_matmul(weights, type, input, output, rows, columns, inner) ? 1 : 0;
}

void pixref_decode(const unsigned char* data, uint32_t type, size_t count, float* output)
{
    cpu_decode(data, type, count, output);
}

uint64_t pixref_weight_bytes(uint64_t inner, uint64_t rows, uint32_t type)
{
    return weight_bytes({inner, rows}, type);
}

void pixref_set_threads(size_t count)
{
    cpu_set_threads(count);
}

size_t pixref_thread_count(void)
{
    return cpu_thread_count();
}

}
