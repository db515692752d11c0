// The lm_head logits without any allocation, for callers that cannot call
// cudaMalloc: a process whose GPU memory belongs to another allocator (a
// framework's caching pool that has reserved nearly all of HBM, where a
// stray cudaMalloc fails or fragments the pool), or a serving loop that must
// not take cudaMalloc's implicit device-wide synchronisation mid-stream.
//
// The A8 activations the matmul reads (int8 rows and their group scales)
// live in one file-scope device array instead of a caller- or
// engine-allocated buffer. Its name in host code is only a host-side
// stand-in, so the first call on each device looks up the array's real
// device address with cudaGetSymbolAddress while that device is current,
// and every later call on that device reuses it.

#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "kernels.h"
#include "needle_engine.h"

namespace nd {

// Defined in engine.cu: the tied lm_head matrix of a loaded model (its
// first out_rows rows).
bool model_head(const nd_model* m, DevMat* emb, int* device, int* out_rows);
void set_error(const std::string& msg);

// At most this many rows per call: 64 x 768 int8 activations plus 64 x 6
// f32 group scales, 50 KB held on every device that loads the library.
constexpr int NOALLOC_MAX_ROWS = 64;
constexpr size_t NOALLOC_ACT_BYTES = (size_t)NOALLOC_MAX_ROWS * 768;
constexpr size_t NOALLOC_BYTES = NOALLOC_ACT_BYTES + (size_t)NOALLOC_MAX_ROWS * 6 * sizeof(float);

static __device__ __align__(256) int8_t g_noalloc_scratch[NOALLOC_BYTES];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[256];  // the array's device address, per device id

// The scratch array's device address on `device` (looked up once, with the
// device current, then cached).
static int8_t* noalloc_scratch(int device) {
    if (device < 0 || device >= 256) throw std::runtime_error("device id out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        int prev = 0;
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
        e = cudaSetDevice(device);
        if (e != cudaSuccess) throw std::runtime_error(std::string("cudaSetDevice: ") + cudaGetErrorString(e));
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        cudaSetDevice(prev);
        if (e != cudaSuccess || !p)
            throw std::runtime_error(std::string("cudaGetSymbolAddress of the scratch array: ") + cudaGetErrorString(e));
        g_noalloc_ptr[device] = p;
    }
    return (int8_t*)g_noalloc_ptr[device];
}

}  // namespace nd

using namespace nd;

extern "C" int nd_head_logits_noalloc(const nd_model* m, const float* h, int rows, float* out, void* stream) {
    try {
        DevMat emb;
        int device = 0, out_rows = 0;
        if (!m || !h || !out) throw std::runtime_error("nd_head_logits_noalloc: null argument");
        if (!model_head(m, &emb, &device, &out_rows)) throw std::runtime_error("nd_head_logits_noalloc: no model");
        if (rows < 1 || rows > NOALLOC_MAX_ROWS)
            throw std::runtime_error("nd_head_logits_noalloc: rows must be in [1, " + std::to_string(NOALLOC_MAX_ROWS) +
                                     "], got " + std::to_string(rows));
        int8_t* scratch = noalloc_scratch(device);
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        cudaStream_t st = (cudaStream_t)stream;
        int8_t* act = scratch;
        float* sx = (float*)(scratch + NOALLOC_ACT_BYTES);
        // every act byte and scale of rows < `rows` is written before the
        // matmul reads it, so nothing in the array has to start at zero
        launch_prep_act(h, 768, 768, rows, act, sx, st);
        cudaError_t e = launch_cq_gemm(emb, act, sx, rows, 1, out, out_rows, 0, st);
        if (e == cudaSuccess) e = cudaGetLastError();
        cudaSetDevice(prev);
        if (e != cudaSuccess) throw std::runtime_error(std::string("nd_head_logits_noalloc: ") + cudaGetErrorString(e));
        return 0;
    } catch (std::exception& ex) {
        set_error(ex.what());
        return -1;
    }
}
