// pxq_pixelina.hpp -- C++ drop-in shim with Pixelina's matmul signatures.
//
// Header-only glue over the C ABI in pxq.h for Pixelina's C++ code; no CUDA
// header is needed on the including side.
//
//   pxq_pixelina::quant_matmul  -- same signature and bool contract as
//       cpu_quant_matmul (src/tensor.h:74, src/kernels_quant.cpp:369-412):
//       true when handled (output written), false where the reference also
//       returns false (unsupported type or shape) so the caller's existing
//       fallback runs.
//   pxq_pixelina::matmul        -- the shape of cpu_matmul / vulkan_matmul
//       (src/model.h:61, src/backend_vulkan.h:139) without the PixModelFile
//       and PixWeight classes: the caller passes the mapped tensor bytes and
//       the weight's identity, which keys the device cache exactly like the
//       Vulkan backend's "file:name:offset:bytes" (src/backend_vulkan.cpp:744).
//       A row view (tensor_linear_rows, src/tensor.cpp:529-544) arrives as a
//       shifted offset and a smaller row count, i.e. as its own cache entry,
//       just as it does in the Vulkan cache.
//
// Both take and return host buffers, like the functions they replace.
#ifndef PXQ_PIXELINA_HPP
#define PXQ_PIXELINA_HPP

#include <cstdint>
#include <string>

#include "pxq.h"

namespace pxq_pixelina {

inline bool quant_matmul(const unsigned char* weights, uint32_t type, const float* input, float* output, size_t rows,
                         size_t columns, size_t inner)
{
    return pxq_quant_matmul(weights, type, input, output, rows, columns, inner) == PXQ_OK;
}

// output[c*rows + r] = dot(weight row r, input row c) for a GGUF tensor of
// shape [inner, rows] whose bytes start at `data` (file.data + weight.offset).
inline bool matmul(const std::string& filename, const std::string& name, uint64_t offset, const unsigned char* data,
                   uint32_t type, uint64_t inner, uint64_t rows, const float* input, size_t columns, float* output)
{
    const uint64_t bytes = pxq_weight_bytes(inner, rows, type);
    if (!bytes || !data || !input || !output || !columns) return false;
    const std::string key = filename + ":" + name + ":" + std::to_string(offset) + ":" + std::to_string(bytes);
    pxq_weight* w = nullptr;
    if (pxq_weight_upload(data, 0, type, inner, rows, key.c_str(), &w) != PXQ_OK) return false;
    return pxq_matmul_host(w, 0, rows, input, columns, output, rows) == PXQ_OK;
}

}  // namespace pxq_pixelina

#endif
