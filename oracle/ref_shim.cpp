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
 * model.cpp for weight_bytes and the GGUF loader, ...).
 */
#include "kernels_quant.cpp"
#include "model.h"
#include "tensor.h"

#include <cstring>

// One tensor of a model file as the reference's loader parsed it.
struct PixrefTensor {
    char name[256];
    uint32_t type;
    uint32_t rank;
    uint64_t shape[5];
    uint64_t offset;
    uint64_t bytes;
};

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

// Open a GGUF file with PixModelFile::open (src/model.cpp:138-251): returns
// its result (0, MODEL_ERROR_OPEN or MODEL_ERROR_FORMAT); on success the
// tensor directory in name order (the std::map's order) goes to `out` (up to
// `cap` entries) and the count to *count, the metadata key count to *keys.
int pixref_gguf_list(const char* path, PixrefTensor* out, size_t cap, size_t* count, size_t* keys)
{
    PixModelFile file;
    const int rc = file.open(path, false);
    *count = 0;
    *keys = 0;
    if (rc) return rc;
    *keys = file.metadata.size();
    for (const auto& entry : file.weights) {
        if (*count < cap) {
            PixrefTensor& t = out[*count];
            std::memset(&t, 0, sizeof(t));
            std::strncpy(t.name, entry.second.name.c_str(), sizeof(t.name) - 1);
            t.type = entry.second.type;
            t.rank = (uint32_t)entry.second.shape.size();
            for (size_t d = 0; d < entry.second.shape.size() && d < 5; d++) t.shape[d] = entry.second.shape[d];
            t.offset = entry.second.offset;
            t.bytes = entry.second.bytes;
        }
        (*count)++;
    }
    return 0;
}

// tensor_attention's range overload (src/tensor.cpp:384-427) on host arrays:
// q [q_rows][heads*d], k, v [k_rows][kv_heads*d], out [q_rows][heads*d].
// Returns 0 when the reference returned an empty tensor (invalid arguments).
int pixref_attention(const float* q, size_t q_rows, const float* k, const float* v, size_t k_rows, size_t heads,
                     size_t kv_heads, size_t head_dim, const size_t* begin, const size_t* end, const size_t* key_end,
                     const int* causal, size_t nranges, size_t query_offset, float* out)
{
    PixTensor tq(q_rows, heads * head_dim), tk(k_rows, kv_heads * head_dim), tv(k_rows, kv_heads * head_dim);
    std::copy(q, q + tq.values.size(), tq.values.begin());
    std::copy(k, k + tk.values.size(), tk.values.begin());
    std::copy(v, v + tv.values.size(), tv.values.begin());
    std::vector<PixAttentionRange> ranges;
    for (size_t i = 0; i < nranges; i++) ranges.push_back({begin[i], end[i], key_end[i], causal[i] != 0});
    PixTensor r = tensor_attention(tq, tk, tv, heads, kv_heads, ranges, query_offset);
    if (r.values.empty()) return 0;
    std::copy(r.values.begin(), r.values.end(), out);
    return 1;
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
