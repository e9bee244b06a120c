// shim_check.cpp -- C++ caller of the drop-in shim, checked against the oracle.
//
// Built and run by tests/test_gpu_cxx_shim.py:
//   g++ -O2 -std=c++17 -I include tests/cxx/shim_check.cpp oracle/pxq_oracle.c \
//       -L pixelina_b200 -lpxq -Wl,-rpath,<abs>/pixelina_b200 -o shim_check
// Exercises pxq_pixelina::quant_matmul (cpu_quant_matmul signature) and
// pxq_pixelina::matmul (cpu_matmul shape, cache key file:name:offset:bytes,
// including a tensor_linear_rows-style row view), and the bool contract.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "pxq_pixelina.hpp"

extern "C" {
void pxo_quantize_row_q8_0(const float* x, uint8_t* y, int64_t k);
int pxo_quant_matmul(const uint8_t* weights, uint32_t type, const float* input, float* output, size_t rows, size_t columns,
                     size_t inner);
}

static uint64_t g_state = 0x9e3779b97f4a7c15ull;
static float gauss()
{
    // sum of uniforms: deterministic, roughly normal
    float s = 0.f;
    for (int i = 0; i < 6; i++) {
        g_state = g_state * 6364136223846793005ull + 1442695040888963407ull;
        s += (float)((g_state >> 40) & 0xffffff) / 16777216.0f;
    }
    return s - 3.0f;
}

static double max_abs_rel(const std::vector<float>& a, const std::vector<float>& b)
{
    double m = 0, d = 0;
    for (size_t i = 0; i < a.size(); i++) {
        m = std::fmax(m, std::fabs((double)b[i]));
        d = std::fmax(d, std::fabs((double)a[i] - (double)b[i]));
    }
    return m > 0 ? d / m : d;
}

int main()
{
    const size_t rows = 96, inner = 1024;
    std::vector<float> wf(rows * inner);
    for (auto& v : wf) v = 0.02f * gauss();
    std::vector<uint8_t> w(rows * inner / 32 * 34);
    for (size_t r = 0; r < rows; r++) pxo_quantize_row_q8_0(&wf[r * inner], &w[r * inner / 32 * 34], (int64_t)inner);
    int failures = 0;
    for (size_t columns : {1, 5, 8, 9, 200}) {
        std::vector<float> x(columns * inner);
        for (auto& v : x) v = gauss();
        std::vector<float> ref(columns * rows), got(columns * rows, NAN);
        pxo_quant_matmul(w.data(), PXQ_TYPE_Q8_0, x.data(), ref.data(), rows, columns, inner);
        if (!pxq_pixelina::quant_matmul(w.data(), PXQ_TYPE_Q8_0, x.data(), got.data(), rows, columns, inner)) {
            printf("quant_matmul columns=%zu not handled: %s\n", columns, pxq_last_error());
            failures++;
        } else if (max_abs_rel(got, ref) > 1e-3) {
            printf("quant_matmul columns=%zu error %g\n", columns, max_abs_rel(got, ref));
            failures++;
        }
        // cpu_matmul shape on a row view: rows [32, 96) of the tensor
        const size_t first = 32, count = rows - first, stride = inner / 32 * 34;
        std::vector<float> vref(columns * count), vgot(columns * count, NAN);
        for (size_t c = 0; c < columns; c++)
            for (size_t r = 0; r < count; r++) vref[c * count + r] = ref[c * rows + first + r];
        if (!pxq_pixelina::matmul("model.gguf", "blk.0.ffn_up.weight.32.64", 4096 + first * stride, w.data() + first * stride,
                                  PXQ_TYPE_Q8_0, inner, count, x.data(), columns, vgot.data())) {
            printf("matmul view columns=%zu failed: %s\n", columns, pxq_last_error());
            failures++;
        } else if (max_abs_rel(vgot, vref) > 1e-3) {
            printf("matmul view columns=%zu error %g\n", columns, max_abs_rel(vgot, vref));
            failures++;
        }
    }
    // the reference's `false` cases stay `false`
    std::vector<float> x(9 * inner, 1.0f), y(9 * rows);
    if (pxq_pixelina::quant_matmul(w.data(), PXQ_TYPE_Q8_0, x.data(), y.data(), rows, 4, 48)) failures++;
    if (pxq_pixelina::quant_matmul(w.data(), 1, x.data(), y.data(), rows, 4, inner)) failures++;
    printf(failures ? "FAIL %d\n" : "OK\n", failures);
    return failures ? 1 : 0;
}
