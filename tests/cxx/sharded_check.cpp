// sharded_check.cpp -- C++ caller of the N-sharded C ABI (pxq_comm_*,
// pxq_sharded_matmul_host), one process per GPU, the way a multi-GPU
// Pixelina host (src/backend_cpu.cpp:103-133) would bind it.
//
// Built and run by tests/test_gpu_cxx_sharded.py:
//   g++ -O2 -std=c++17 -I include tests/cxx/sharded_check.cpp oracle/pxq_oracle.c \
//       -L pixelina_b200 -lpxq -Wl,-rpath,<abs>/pixelina_b200 -o sharded_check
//   sharded_check <world> <rank> <id file>      (one process per rank)
// Rank 0 creates the communicator id and publishes it through the id file;
// every rank uploads its share of the weight rows, runs the sharded product
// with host buffers, and compares the whole output bit for bit with the
// single-GPU pxq_quant_matmul of the whole weight.  Prints "OK rank <r>".
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "pxq.h"

extern "C" {
void pxo_quantize_row_q8_0(const float* x, uint8_t* y, int64_t k);
}

static uint64_t g_state = 0x2545f4914f6cdd1dull;
static float gauss()
{
    float s = 0.f;
    for (int i = 0; i < 6; i++) {
        g_state = g_state * 6364136223846793005ull + 1442695040888963407ull;
        s += (float)((g_state >> 40) & 0xffffff) / 16777216.0f;
    }
    return s - 3.0f;
}

static int fail(const char* what, int rc)
{
    std::printf("FAIL %s: rc %d (%s)\n", what, rc, pxq_last_error());
    return 1;
}

int main(int argc, char** argv)
{
    if (argc < 4) {
        std::printf("usage: sharded_check <world> <rank> <id file>\n");
        return 2;
    }
    const int world = std::atoi(argv[1]), rank = std::atoi(argv[2]);
    const std::string id_path = argv[3];
    if (int rc = pxq_init(rank)) return fail("pxq_init", rc);

    // the communicator id: rank 0 writes it (renamed into place), the others wait for it
    unsigned char id[PXQ_COMM_ID_BYTES];
    if (rank == 0) {
        if (int rc = pxq_comm_unique_id(id)) return fail("pxq_comm_unique_id", rc);
        const std::string tmp = id_path + ".tmp";
        FILE* f = std::fopen(tmp.c_str(), "wb");
        if (!f || std::fwrite(id, 1, sizeof(id), f) != sizeof(id)) return fail("write id", -1);
        std::fclose(f);
        std::rename(tmp.c_str(), id_path.c_str());
    } else {
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            FILE* f = std::fopen(id_path.c_str(), "rb");
            if (f && std::fread(id, 1, sizeof(id), f) == sizeof(id)) {
                std::fclose(f);
                break;
            }
            if (f) std::fclose(f);
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60)) return fail("id file", -1);
            std::this_thread::sleep_for(std::chrono::milliseconds(20));
        }
    }
    pxq_comm* comm = nullptr;
    if (int rc = pxq_comm_init(id, world, rank, 60000, &comm)) return fail("pxq_comm_init", rc);

    // the same Q8_0 weight and activation on every rank
    const size_t rows = 512, inner = 1024, row_bytes = inner / 32 * 34;
    std::vector<uint8_t> w(rows * row_bytes);
    {
        std::vector<float> wf(inner);
        for (size_t r = 0; r < rows; r++) {
            for (auto& v : wf) v = 0.02f * gauss();
            pxo_quantize_row_q8_0(wf.data(), &w[r * row_bytes], (int64_t)inner);
        }
    }
    int bad = 0;
    for (size_t columns : {size_t(200), size_t(9)}) {
        std::vector<float> x(columns * inner);
        for (auto& v : x) v = gauss();
        std::vector<float> ref(columns * rows), got(columns * rows, -1.f);
        if (int rc = pxq_quant_matmul(w.data(), PXQ_TYPE_Q8_0, x.data(), ref.data(), rows, columns, inner))
            return fail("pxq_quant_matmul", rc);
        const size_t shard = rows / (size_t)world;
        pxq_weight* ws = nullptr;
        if (int rc = pxq_weight_upload(&w[(size_t)rank * shard * row_bytes], 0, PXQ_TYPE_Q8_0, inner, shard, nullptr, &ws))
            return fail("pxq_weight_upload", rc);
        for (int call = 0; call < 2; call++) {
            if (int rc = pxq_sharded_matmul_host(comm, ws, shard, x.data(), columns, inner, got.data()))
                return fail("pxq_sharded_matmul_host", rc);
            if (std::memcmp(got.data(), ref.data(), got.size() * sizeof(float)) != 0) {
                std::printf("DIFFERENT rank %d columns %zu call %d\n", rank, columns, call);
                bad++;
            }
        }
        pxq_weight_release(ws);
    }
    if (int rc = pxq_comm_barrier(comm)) return fail("pxq_comm_barrier", rc);
    pxq_comm_destroy(comm);
    if (bad) return 1;
    std::printf("OK rank %d of %d\n", rank, world);
    return 0;
}
