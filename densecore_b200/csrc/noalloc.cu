// noalloc.cu -- dcg_mul_mat_noalloc: the quantized matmul without any caller-provided or
// library-allocated scratch.
//
// Some callers cannot allocate device memory at the point where they run the matmul: a ggml
// custom-op callback runs inside the graph-compute thread pool with no allocator handle, plugin
// hosts may forbid cudaMalloc after start-up, and allocation can synchronize the device in the
// middle of a step.  This entry point keeps the quantized activation in a fixed, file-scope device
// array instead, so it calls no cudaMalloc / cudaFree (and no allocating library routine).
//
// Limits and sharing rules:
//   * the array holds NOALLOC_SCRATCH_BYTES (1 MiB) on every GPU that loads the library, until the
//     process exits; calls whose activation needs more (dcg_act_size) are rejected with DCG_EINVAL;
//   * every call uses the same array and leaves its contents behind.  The quantize kernel rewrites
//     every byte the GEMV later reads, so nothing has to start at zero;
//   * calls whose work overlaps on the GPU (different streams, or other threads on the same
//     device) race on the array: serialize them on one stream;
//   * the first call on each device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current; make that first call before any stream capture.
#include <mutex>
#include <string>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"

namespace dcg_internal {
void set_error(const std::string& m);
}

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(1) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void* g_dev_ptr[MAX_DEVICES] = {};

int nfail(int code, const std::string& m) {
    dcg_internal::set_error(m);
    return code;
}

// device address of g_noalloc_scratch on the current device (looked up once per device)
int scratch_ptr(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return nfail(DCG_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= MAX_DEVICES) return nfail(DCG_EINVAL, "device index out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dev_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return nfail(DCG_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_dev_ptr[dev] = p;
    }
    *out = g_dev_ptr[dev];
    return DCG_OK;
}

}  // namespace

extern "C" int dcg_mul_mat_noalloc(int type, const void* w, int64_t n, int64_t k, const float* x,
                                   int64_t m, float* y, void* stream) {
    if (type != DCG_TYPE_Q8_0 && type != DCG_TYPE_Q4_K && type != DCG_TYPE_Q6_K)
        return nfail(DCG_EINVAL, "unsupported weight type " + std::to_string(type));
    const int64_t blk = type == DCG_TYPE_Q8_0 ? QK8_0 : QK_K;
    if (n < 0 || m < 0 || k <= 0 || k % blk) return nfail(DCG_EINVAL, "bad shape");
    if (m == 0 || n == 0) return DCG_OK;
    if (!w || !x || !y) return nfail(DCG_EINVAL, "null pointer");
    if ((uintptr_t)w % 256 || (uintptr_t)x % 16 || (uintptr_t)y % 4)
        return nfail(DCG_EINVAL, "w must be 256-byte, x 16-byte and y 4-byte aligned");
    const int act_type = type == DCG_TYPE_Q8_0 ? DCG_TYPE_Q8_0 : DCG_TYPE_Q8_K;
    const size_t need = dcg::act_bytes(act_type, m, k);
    if (need > NOALLOC_SCRATCH_BYTES)
        return nfail(DCG_EINVAL, "activation of m=" + std::to_string(m) + " x k=" + std::to_string(k) +
                                     " needs " + std::to_string(need) + " bytes of scratch; the fixed "
                                     "no-allocation buffer holds " + std::to_string(NOALLOC_SCRATCH_BYTES));
    void* scratch = nullptr;
    int rc = scratch_ptr(&scratch);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = dcg::launch_quantize_act(act_type, x, scratch, m, k, true, st);
    for (int64_t m0 = 0; e == cudaSuccess && m0 < m; m0 += 8) {
        const int64_t mc = (m - m0) < 8 ? (m - m0) : 8;
        e = dcg::launch_gemv(type, w, n, k, scratch, m, m0, mc, y, st);
    }
    if (e != cudaSuccess) return nfail(DCG_ECUDA, std::string("mul_mat_noalloc: ") + cudaGetErrorString(e));
    return DCG_OK;
}
