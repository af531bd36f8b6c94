// ctx.cu -- host-boundary entry points (dcg_ctx_*): one context per device that owns a stream,
// the resident weights (keyed by the caller's host pointer, i.e. ggml tensor->data), a growable
// scratch/activation buffer and pinned staging memory.  Declarations: include/dcgpu.h.
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <cstring>

#include "../../include/dcgpu.h"
#include "common.cuh"
#include "kernels.h"

struct dcg_weight {
    int type;
    int64_t n, k;
    void* dev;  // packed device layout
    const void* host_key;
};

struct dcg_ctx {
    int device;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::unordered_map<const void*, dcg_weight*> by_host;
    void* scratch = nullptr;  // device: [activation f32 | quantized activation | output f32]
    size_t scratch_cap = 0;
    void* pinned = nullptr;  // host staging, same layout as the f32 parts (mapped into the device)
    void* pinned_dev = nullptr;  // its device address
    size_t pinned_cap = 0;
};

// the per-thread message store lives in capi.cu
namespace dcg_internal {
void set_error(const std::string& m);
}

namespace {
int ctx_fail(int code, const std::string& m) {
    dcg_internal::set_error(m);
    return code;
}
int cerr(cudaError_t e, const char* where) {
    return ctx_fail(e == cudaErrorMemoryAllocation ? DCG_ENOMEM : DCG_ECUDA,
                    std::string(where) + ": " + cudaGetErrorString(e));
}
#define CTX_CUDA(call, where)                         \
    do {                                              \
        cudaError_t _e = (call);                      \
        if (_e != cudaSuccess) return cerr(_e, where); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int grow(dcg_ctx* c, size_t dev_bytes, size_t host_bytes) {
    if (dev_bytes > c->scratch_cap) {
        if (c->scratch) cudaFree(c->scratch);
        c->scratch = nullptr;
        c->scratch_cap = 0;
        CTX_CUDA(cudaMalloc(&c->scratch, dev_bytes), "cudaMalloc(scratch)");
        c->scratch_cap = dev_bytes;
    }
    if (host_bytes > c->pinned_cap) {
        if (c->pinned) cudaFreeHost(c->pinned);
        c->pinned = nullptr;
        c->pinned_cap = 0;
        CTX_CUDA(cudaHostAlloc(&c->pinned, host_bytes, cudaHostAllocMapped), "cudaHostAlloc(staging)");
        const cudaError_t e = cudaHostGetDevicePointer(&c->pinned_dev, c->pinned, 0);
        if (e != cudaSuccess) {
            cudaFreeHost(c->pinned);
            c->pinned = nullptr;
            return cerr(e, "cudaHostGetDevicePointer(staging)");
        }
        c->pinned_cap = host_bytes;
    }
    return DCG_OK;
}
}  // namespace

extern "C" {

int dcg_ctx_create(int device, dcg_ctx** out) {
    if (!out) return ctx_fail(DCG_EINVAL, "null out");
    int ndev = 0;
    CTX_CUDA(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
    if (device < 0 || device >= ndev) return ctx_fail(DCG_EINVAL, "no such device");
    DeviceGuard g(device);
    auto c = std::make_unique<dcg_ctx>();
    c->device = device;
    CTX_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    *out = c.release();
    return DCG_OK;
}

int dcg_ctx_destroy(dcg_ctx* c) {
    if (!c) return DCG_OK;
    {
        DeviceGuard g(c->device);
        std::lock_guard<std::mutex> lk(c->mu);
        cudaStreamSynchronize(c->stream);
        for (auto& kv : c->by_host) {
            cudaFree(kv.second->dev);
            delete kv.second;
        }
        c->by_host.clear();
        if (c->scratch) cudaFree(c->scratch);
        if (c->pinned) cudaFreeHost(c->pinned);
        cudaStreamDestroy(c->stream);
    }
    delete c;
    return DCG_OK;
}

int dcg_ctx_weight_register(dcg_ctx* c, int type, const void* host_rows, size_t row_stride,
                            int64_t n, int64_t k, dcg_weight** out) {
    if (!c || !host_rows || !out) return ctx_fail(DCG_EINVAL, "null pointer");
    if (type != DCG_TYPE_Q8_0 && type != DCG_TYPE_Q4_K && type != DCG_TYPE_Q6_K)
        return ctx_fail(DCG_EINVAL, "unsupported weight type");
    const int64_t blk = type == DCG_TYPE_Q8_0 ? QK8_0 : QK_K;
    if (n <= 0 || k <= 0 || k % blk) return ctx_fail(DCG_EINVAL, "bad shape");
    const size_t rs = dcg_row_size(type, k);
    if (row_stride < rs) return ctx_fail(DCG_EINVAL, "row_stride smaller than a row");
    DeviceGuard g(c->device);
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->by_host.count(host_rows)) {
        dcg_weight* old = c->by_host[host_rows];
        if (old->type != type || old->n != n || old->k != k)
            return ctx_fail(DCG_EINVAL, "host pointer already registered as a different weight (type/n/k); "
                                        "release it first");
        *out = old;
        return DCG_OK;
    }
    void* raw = nullptr;
    void* dev = nullptr;
    CTX_CUDA(cudaMalloc(&raw, rs * (size_t)n), "cudaMalloc(upload)");
    cudaError_t e = cudaMemcpy2DAsync(raw, rs, host_rows, row_stride, rs, (size_t)n,
                                      cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMalloc(&dev, dcg::packed_weight_bytes(type, n, k));
    if (e == cudaSuccess) e = dcg::launch_pack(type, raw, rs, dev, n, k, false, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(raw);
    if (e != cudaSuccess) {
        if (dev) cudaFree(dev);
        return cerr(e, "weight upload");
    }
    auto* w = new dcg_weight{type, n, k, dev, host_rows};
    c->by_host[host_rows] = w;
    *out = w;
    return DCG_OK;
}

int dcg_ctx_weight_release(dcg_ctx* c, dcg_weight* w) {
    if (!c || !w) return ctx_fail(DCG_EINVAL, "null pointer");
    DeviceGuard g(c->device);
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->by_host.find(w->host_key);
    if (it == c->by_host.end() || it->second != w) return ctx_fail(DCG_ENOTFOUND, "weight not registered");
    c->by_host.erase(it);
    cudaStreamSynchronize(c->stream);
    cudaFree(w->dev);
    delete w;
    return DCG_OK;
}

int dcg_ctx_find_weight(dcg_ctx* c, const void* host_rows, dcg_weight** out) {
    if (!c || !out) return ctx_fail(DCG_EINVAL, "null pointer");
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->by_host.find(host_rows);
    if (it == c->by_host.end()) return ctx_fail(DCG_ENOTFOUND, "host pointer not registered");
    *out = it->second;
    return DCG_OK;
}

int dcg_ctx_mul_mat(dcg_ctx* c, dcg_weight* w, const float* x_host, int64_t m, float* y_host) {
    if (!c || !w || !x_host || !y_host) return ctx_fail(DCG_EINVAL, "null pointer");
    if (m <= 0) return m == 0 ? DCG_OK : ctx_fail(DCG_EINVAL, "m < 0");
    DeviceGuard g(c->device);
    std::lock_guard<std::mutex> lk(c->mu);
    const size_t xb = dcg::align256((size_t)m * w->k * 4), yb = dcg::align256((size_t)m * w->n * 4);
    const size_t qb = dcg_mul_mat_scratch_size(w->type, w->n, w->k, m);
    int rc = grow(c, xb + qb + yb, xb + yb);
    if (rc) return rc;
    uint8_t* dx = (uint8_t*)c->scratch;
    uint8_t* dq = dx + xb;
    uint8_t* dy = dq + qb;
    uint8_t* hx = (uint8_t*)c->pinned;
    uint8_t* hy = hx + xb;
    memcpy(hx, x_host, (size_t)m * w->k * 4);
    CTX_CUDA(cudaMemcpyAsync(dx, hx, (size_t)m * w->k * 4, cudaMemcpyHostToDevice, c->stream), "H2D");
    // m = 1: the kernel writes y straight into the mapped staging buffer (one row of posted PCIe
    // writes), so no device-to-host copy follows; larger m go through device memory and a copy
    float* ydst = m == 1 ? (float*)((uint8_t*)c->pinned_dev + xb) : (float*)dy;
    rc = dcg_mul_mat(w->type, w->dev, w->n, w->k, (const float*)dx, m, ydst, dq, qb, c->stream);
    if (rc) return rc;
    if (m != 1)
        CTX_CUDA(cudaMemcpyAsync(hy, dy, (size_t)m * w->n * 4, cudaMemcpyDeviceToHost, c->stream), "D2H");
    CTX_CUDA(cudaStreamSynchronize(c->stream), "sync");
    memcpy(y_host, hy, (size_t)m * w->n * 4);
    return DCG_OK;
}

}  // extern "C"
