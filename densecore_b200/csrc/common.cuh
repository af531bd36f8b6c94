// common.cuh -- shared definitions for the dcgpu sm_100a kernels.
//
// Block formats are ggml's (GGUF): Q8_0 (32 x int8 + fp16 d, 34 B), Q4_K (256: fp16 d, fp16 dmin,
// 12 B packed 6-bit scales/mins, 128 B nibbles; 144 B), Q6_K (256: 128 B low nibbles, 64 B high
// 2-bit planes, 16 int8 scales, fp16 d; 210 B), Q8_K (256: f32 d, 256 int8, 16 int16 bsums; 292 B).
//
// Device ("packed") weight layout, written once at upload by dcg_weight_pack:
//   Q4_K : unchanged ggml rows (a 144-B block is nine 16-B vectors).
//   Q8_0 : payload [n][k] int8 (row = k bytes), then fp16 d [n][k/32].
//   Q6_K : payload [n][k/256][208 B = ql|qh|scales], then fp16 d [n][k/256].
// Device activation layout (written by the quantize kernels for mul_mat):
//   Q8_0 act : qs [m][k] int8, then fp16 d [m][k/32].
//   Q8_K act : qs [m][k] int8, then f32 d [m][k/256], then int16 bsums [m][k/16], then int16
//              bsums32 [m][k/32] (sums of 32: bsums[2j] + bsums[2j+1], the Q4_K min-term operand).
// Every region starts on a 256-B boundary so every payload load is an aligned 16-B vector.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#define DCG_TYPE_F32 0
#define DCG_TYPE_F16 1
#define DCG_TYPE_Q8_0 8
#define DCG_TYPE_Q4_K 12
#define DCG_TYPE_Q6_K 14
#define DCG_TYPE_Q8_K 15

#define QK8_0 32
#define QK_K 256
#define Q8_0_BYTES 34
#define Q4_K_BYTES 144
#define Q6_K_BYTES 210
#define Q6_K_PAYLOAD 208
#define Q8_K_BYTES 292

namespace dcg {

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- packed weight layout ----
struct PackedW {
    const uint8_t* payload;  // row-major payload
    const __half* d;         // per-block fp16 scales (Q8_0, Q6_K); null for Q4_K
    size_t row_bytes;        // payload bytes per row
    int nb;                  // blocks per row (32-blocks for Q8_0, 256-blocks for K-quants)
};

__host__ __device__ inline size_t packed_payload_row_bytes(int type, int64_t k) {
    switch (type) {
        case DCG_TYPE_Q8_0: return (size_t)k;
        case DCG_TYPE_Q4_K: return (size_t)(k / QK_K) * Q4_K_BYTES;
        case DCG_TYPE_Q6_K: return (size_t)(k / QK_K) * Q6_K_PAYLOAD;
    }
    return 0;
}
__host__ __device__ inline int blocks_per_row(int type, int64_t k) {
    return type == DCG_TYPE_Q8_0 ? (int)(k / QK8_0) : (int)(k / QK_K);
}
__host__ __device__ inline size_t packed_weight_bytes(int type, int64_t n, int64_t k) {
    size_t p = align256(packed_payload_row_bytes(type, k) * (size_t)n);
    if (type == DCG_TYPE_Q4_K) return p;
    return p + align256((size_t)n * blocks_per_row(type, k) * 2);
}
__host__ __device__ inline PackedW packed_view(int type, const void* base, int64_t n, int64_t k) {
    PackedW w;
    w.payload = (const uint8_t*)base;
    w.row_bytes = packed_payload_row_bytes(type, k);
    w.nb = blocks_per_row(type, k);
    w.d = type == DCG_TYPE_Q4_K ? nullptr
                                : (const __half*)(w.payload + align256(w.row_bytes * (size_t)n));
    return w;
}

// ---- activation layout ----
struct ActQ {
    int8_t* qs;      // [m][k]
    void* d;         // fp16 [m][k/32] (Q8_0) or f32 [m][k/256] (Q8_K)
    int16_t* bsums;  // [m][k/16] (Q8_K only)
    int16_t* bs32;   // [m][k/32] (Q8_K only)
};
__host__ __device__ inline size_t act_bytes(int act_type, int64_t m, int64_t k) {
    size_t q = align256((size_t)m * k);
    if (act_type == DCG_TYPE_Q8_0) return q + align256((size_t)m * (k / QK8_0) * 2);
    return q + align256((size_t)m * (k / QK_K) * 4) + align256((size_t)m * (k / 16) * 2) +
           align256((size_t)m * (k / 32) * 2);
}
__host__ __device__ inline ActQ act_view(int act_type, void* base, int64_t m, int64_t k) {
    ActQ a;
    uint8_t* p = (uint8_t*)base;
    a.qs = (int8_t*)p;
    p += align256((size_t)m * k);
    a.d = p;
    if (act_type == DCG_TYPE_Q8_0) {
        a.bsums = nullptr;
        a.bs32 = nullptr;
    } else {
        p += align256((size_t)m * (k / QK_K) * 4);
        a.bsums = (int16_t*)p;
        p += align256((size_t)m * (k / 16) * 2);
        a.bs32 = (int16_t*)p;
    }
    return a;
}

// ---- loads ----
// Streaming 16-B weight load: read-only path, no L1 allocation, 256-B L2 prefetch.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
// Activation load: cached in L1 (every warp of the SM reads the same activation rows).
__device__ __forceinline__ uint4 ld_act_v4(const void* p) { return __ldg((const uint4*)p); }

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// 6-bit scale/min j (0..7) from the 12-byte Q4_K scale field given as three u32 words
// (bytes 0-3, 4-7, 8-11); ggml's get_scale_min_k4 bit layout.
// the 6-bit scales (sc) and mins (mn) of Q4_K sub-blocks 0-3 / 4-7, one per byte, from the block's
// first 16 bytes (d, dmin, 12 packed scale bytes)
struct Q4kScales {
    uint32_t sc03, sc47, mn03, mn47;
};
__device__ __forceinline__ Q4kScales q4k_unpack(const uint4& h) {
    Q4kScales s;
    s.sc03 = h.y & 0x3F3F3F3Fu;
    s.mn03 = h.z & 0x3F3F3F3Fu;
    s.sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    s.mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    return s;
}

__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc,
                                              int& m) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63;
        m = (s1 >> (8 * j)) & 63;
    } else {
        const int jj = j - 4;
        const uint32_t b8 = (s2 >> (8 * jj)) & 0xFF;
        sc = (b8 & 0xF) | (((s0 >> (8 * jj + 6)) & 3) << 4);
        m = (b8 >> 4) | (((s1 >> (8 * jj + 6)) & 3) << 4);
    }
}

// ---- programmatic dependent launch (PDL) ----
// pdl_wait: block until the grid this one depends on has completed and its writes are visible
// (a no-op when the kernel was not launched as a programmatic dependent).  pdl_trigger: allow the
// next kernel in the stream to start launching.  Every kernel here calls pdl_wait before it reads
// or writes any buffer another kernel produces or consumes; only constant weights are touched
// before it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Process-wide switch for programmatic dependent launch (dcg_set_programmatic_launch).  When off,
// every launch is plainly stream-ordered: a kernel starts only after its predecessor in the stream
// has completed, whatever that predecessor is (a collective or another library's kernel included).
inline std::atomic<int>& pdl_flag() {
    static std::atomic<int> flag{1};
    return flag;
}

// Launch with optional thread-block cluster (cluster_z CTAs along z; 1 = no cluster) and, when the
// switch above is on, the programmatic-stream-serialization attribute (the kernel may start while
// its predecessor drains; it reads the predecessor's outputs only after pdl_wait).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, unsigned cluster_z, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (cluster_z > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = cluster_z;
        na++;
    }
    if (pdl_flag().load(std::memory_order_relaxed)) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
    return launch_ex(kernel, grid, block, smem, st, 1u, std::forward<Args>(args)...);
}

// ---- per-device one-time setup ----
// Kernel attributes (cudaFuncSetAttribute) and device properties are per device; a process may drive
// several GPUs from several threads.  per_device_once runs `fn` once for the calling thread's current
// device and returns its (cached) result.
constexpr int MAX_DEVICES = 64;
struct PerDevice {
    std::once_flag once[MAX_DEVICES];
    cudaError_t err[MAX_DEVICES] = {};
};
template <class F>
inline cudaError_t per_device_once(PerDevice& pd, F&& fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
    std::call_once(pd.once[dev], [&] { pd.err[dev] = fn(); });
    return pd.err[dev];
}
// dynamic shared memory opt-in of `kernel` on the current device (once per device)
#define DCG_SMEM_ATTR(kernel, bytes)                                                               \
    ([&]() -> cudaError_t {                                                                        \
        static ::dcg::PerDevice pd_;                                                               \
        return ::dcg::per_device_once(pd_, [&] {                                                   \
            return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(bytes)); \
        });                                                                                        \
    }())
// streaming multiprocessors of the current device (cached per device)
inline int num_sms() {
    static int sms[MAX_DEVICES] = {};
    static PerDevice pd;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return 148;
    per_device_once(pd, [&] {
        int v = 0;
        cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = v > 0 ? v : 148;
        return e;
    });
    return sms[dev];
}

}  // namespace dcg
