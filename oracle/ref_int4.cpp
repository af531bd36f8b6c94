// Timing wrapper around DenseCore's own INT4 decode GEMV (core/src/kernels/cpu_int4.cpp:1404-1443,
// GemvInt4 with its runtime ISA dispatch: AVX512-VNNI, AVX-512, AVX2).  Off the GGUF path: its
// weights are DenseCore's custom INT4 layout (K/2 packed nibbles per row, an f32 scale and zero per
// group), so it is reported beside the CPU baseline as the reference's own best-ISA integer GEMV,
// not as a parity oracle.  Test / measurement infrastructure only.
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <thread>
#include <vector>

#include "kernels/cpu_int4.h"

extern "C" const char* ref_int4_isa() {
    if (__builtin_cpu_supports("avx512vnni")) return "avx512vnni";
    if (__builtin_cpu_supports("avx512f")) return "avx512f";
    if (__builtin_cpu_supports("avx2")) return "avx2";
    return "none";
}

// Repeats y = W x over the (n, k) matrices for about `budget_s` seconds on `threads` threads
// (output rows split into contiguous slices, as cb_gemv_custom does); returns the number of full
// passes and writes the elapsed seconds.
extern "C" long ref_int4_time(const int* ns, const int* ks, int nmat, int group, int threads, double budget_s,
                              double* seconds) {
    struct Mat {
        int n, k;
        std::vector<uint8_t> w;
        std::vector<float> s, z, x, y;
    };
    std::vector<Mat> mats(nmat);
    uint32_t st = 12345u;
    auto rnd = [&]() { st = st * 1664525u + 1013904223u; return st; };
    for (int i = 0; i < nmat; i++) {
        Mat& m = mats[i];
        m.n = ns[i];
        m.k = ks[i];
        m.w.resize((size_t)m.n * m.k / 2);
        for (auto& b : m.w) b = (uint8_t)(rnd() >> 24);
        const size_t ng = (size_t)m.n * (m.k / group);
        m.s.assign(ng, 0.01f);
        m.z.assign(ng, 8.0f);
        m.x.resize(m.k);
        for (auto& v : m.x) v = (float)((int)(rnd() >> 16) % 2001 - 1000) * 1e-3f;
        m.y.assign(m.n, 0.0f);
    }
    long passes = 0;
    const auto t0 = std::chrono::steady_clock::now();
    double el = 0.0;
    do {
        for (Mat& m : mats) {
            std::vector<std::thread> pool;
            const int per = (m.n + threads - 1) / threads;
            for (int t = 0; t < threads; t++) {
                const int a = t * per, b = a + per < m.n ? a + per : m.n;
                if (a >= b) break;
                pool.emplace_back([&m, a, b, group] {
                    densecore::kernels::GemvInt4(m.y.data(), m.x.data(), m.w.data(), m.s.data(), m.z.data(), m.k,
                                                 m.n, group, a, b);
                });
            }
            for (auto& th : pool) th.join();
        }
        passes++;
        el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    } while (el < budget_s);
    *seconds = el;
    return passes;
}
