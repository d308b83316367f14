// Shared pieces of the command-line drivers (one binary per kernel family, same flags and
// stdout lines as the reference's OpenCL drivers, int2_fp16_upcvt/main.cpp:378-431 and
// siblings, so the reference's bench / validate scripts can run them unchanged):
//   - fp16 / bf16 raw-bit conversions (round to nearest even; bf16 NaN quieted),
//   - the fused epilogue on the host gold and the pass rules of the reference drivers
//     (per element |d| <= abs_tol || ulp <= ulp_tol || rel <= 1e-3; fp32 outputs
//     |d| <= 0.05 || rel <= 2e-4; common/epilogue.hpp, int2_fp16_upcvt/main.cpp:100-121),
//   - device buffers, CUDA-event timing and the flag parser.
// The drivers call libternocl through its C ABI only (include/ternocl.h).
#pragma once

#include <cuda_runtime.h>
#include <omp.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <random>
#include <string>
#include <vector>

#include "ternocl.h"

namespace drv {

constexpr int kGS = 128;

// ---- 16-bit activation / scale / output type ------------------------------------------
inline bool &bf16_mode() {
    static bool v = false;
    return v;
}
inline const char *dt_name() { return bf16_mode() ? "bf16" : "fp16"; }
inline int dt_code() { return bf16_mode() ? TERNOCL_BF16 : TERNOCL_FP16; }

inline float bits_to_f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline uint32_t f_to_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
inline float tof(uint16_t h) {
    if (bf16_mode()) return bits_to_f((uint32_t)h << 16);
    _Float16 x;
    std::memcpy(&x, &h, 2);
    return (float)x;
}
inline uint16_t fromf(float f) {
    if (bf16_mode()) {
        const uint32_t u = f_to_bits(f);
        if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  // quiet NaN
        const uint32_t lsb = (u >> 16) & 1u;
        return (uint16_t)((u + 0x7fffu + lsb) >> 16);
    }
    const _Float16 x = (_Float16)f;
    uint16_t h;
    std::memcpy(&h, &x, 2);
    return h;
}

// ---- random inputs ----------------------------------------------------------------------
// Seeded from --seed when given, else from std::random_device (as the reference drivers).
inline uint64_t &seed_base() {
    static uint64_t s = 0;
    return s;
}
inline bool &seed_fixed() {
    static bool v = false;
    return v;
}
inline std::mt19937_64 &thread_rng() {
    static thread_local std::mt19937_64 g([]() -> uint64_t {
        const uint64_t t = (uint64_t)omp_get_thread_num();
        if (seed_fixed()) return seed_base() * 0x9E3779B97F4A7C15ull + t + 1;
        return ((uint64_t)std::random_device{}() << 32) ^ (uint64_t)std::random_device{}() ^ t;
    }());
    return g;
}
inline uint32_t rnd_u32() { return (uint32_t)(thread_rng()() >> 32); }
inline float rnd_uniform(float lo, float hi) {
    return lo + (hi - lo) * (float)((thread_rng()() >> 40) * (1.0 / 16777216.0));
}
// ternary int2 word: codes {0, 1, 3} = {0, +1, -1} with P(0) = 1/2
inline uint32_t rnd_int2_word() {
    const uint32_t a = rnd_u32(), b = rnd_u32();
    return (a & 0x55555555u) | ((a & b & 0x55555555u) << 1);
}
inline int int2_code_value(uint32_t c) { return c == 1 ? 1 : c == 3 ? -1 : c == 2 ? -2 : 0; }

// ---- epilogue -----------------------------------------------------------------------------
struct Epilogue {
    int postop = 0;  // 0 none, 1 silu(acc)*other, 2 acc+other, 3 acc+bias[n], 4 sigmoid(acc)
    bool out_f32 = false;
    bool needs_other() const { return postop == 1 || postop == 2; }
    bool needs_bias() const { return postop == 3; }
    size_t out_size() const { return out_f32 ? 4 : 2; }
    std::string name() const {
        static const char *n[] = {"none", "silu(acc)*other", "acc+other", "acc+bias", "sigmoid(acc)"};
        return std::string(n[postop]) + (out_f32 ? ", fp32 out" : "");
    }
    // sigmoid lies in (0, 1): its absolute bound is on that scale
    double abs_tol() const {
        if (postop == 4) return bf16_mode() && !out_f32 ? 0.03 : 0.004;
        return bf16_mode() ? 16.0 : 8.0;
    }
    uint32_t ulp_tol() const { return postop == 4 ? 4u : (bf16_mode() ? 32u : 64u); }
};

inline float sigmoid_host(float x) { return x <= -10.0f ? 0.0f : 1.0f / (1.0f + std::exp(-x)); }

// Other ~ U(-4, 4) [M, N] DT; Bias ~ U(-8, 8) [N] DT or fp32
inline void fill_epilogue_inputs(const Epilogue &e, std::vector<uint16_t> &other, std::vector<unsigned char> &bias,
                                 int M, int N) {
    other.assign(e.needs_other() ? (size_t)M * N : 0, 0);
    for (auto &o : other) o = fromf(rnd_uniform(-4.0f, 4.0f));
    bias.assign(e.needs_bias() ? (size_t)N * e.out_size() : 0, 0);
    for (int n = 0; e.needs_bias() && n < N; ++n) {
        const float b = rnd_uniform(-8.0f, 8.0f);
        if (e.out_f32) std::memcpy(&bias[4 * (size_t)n], &b, 4);
        else {
            const uint16_t h = fromf(b);
            std::memcpy(&bias[2 * (size_t)n], &h, 2);
        }
    }
}

// out = cast(epi(acc)) for the fp32 gold accumulators
inline void apply_epilogue(const Epilogue &e, const float *acc, const uint16_t *other, const unsigned char *bias,
                           unsigned char *out, int M, int N) {
#pragma omp parallel for
    for (long long i = 0; i < (long long)M * N; ++i) {
        float v = acc[i];
        const size_t n = (size_t)(i % N);
        switch (e.postop) {
            case 1: v = v * sigmoid_host(v) * tof(other[i]); break;
            case 2: v += tof(other[i]); break;
            case 3: {
                float b;
                if (e.out_f32) std::memcpy(&b, bias + 4 * n, 4);
                else {
                    uint16_t h;
                    std::memcpy(&h, bias + 2 * n, 2);
                    b = tof(h);
                }
                v += b;
                break;
            }
            case 4: v = sigmoid_host(v); break;
            default: break;
        }
        if (e.out_f32) std::memcpy(out + 4 * (size_t)i, &v, 4);
        else {
            const uint16_t h = fromf(v);
            std::memcpy(out + 2 * (size_t)i, &h, 2);
        }
    }
}

// ---- pass rules ---------------------------------------------------------------------------
inline bool compare_dt(const uint16_t *C, const uint16_t *G, size_t n, const std::string &label, double abs_tol,
                       uint32_t ulp_tol) {
    size_t bad = 0, ulp_at = 0, abs_at = 0;
    uint32_t ulp_max = 0;
    double abs_max = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const uint32_t ulp = C[i] > G[i] ? C[i] - G[i] : G[i] - C[i];
        const float got = tof(C[i]), want = tof(G[i]);
        const double d = std::fabs((double)got - want);
        if (ulp > ulp_max) ulp_max = ulp, ulp_at = i;
        if (d > abs_max || std::isnan(d)) abs_max = d, abs_at = i;
        const bool ok = d <= abs_tol || ulp <= ulp_tol || std::fabs((want - got) / want) <= 0.001;
        if (!ok && ++bad <= 10) std::cout << "\tidx " << i << " data " << got << " gold " << want << "\n";
    }
    std::cout << label << ": max abs diff " << abs_max << " (idx " << abs_at << "), max ULP diff " << ulp_max
              << " (idx " << ulp_at << "), pass rate " << 100.0 * (double)(n - bad) / (double)n << "%\n";
    return bad == 0;
}

inline bool compare_f32(const float *C, const float *G, size_t n, const std::string &label) {
    size_t bad = 0;
    double abs_max = 0.0, rel_max = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double d = std::fabs((double)C[i] - G[i]);
        const double r = d / std::max(1e-30, (double)std::fabs(G[i]));
        abs_max = std::max(abs_max, std::isnan(d) ? INFINITY : d);
        rel_max = std::max(rel_max, std::isnan(r) ? INFINITY : r);
        if (!(d <= 0.05 || r <= 2e-4) && ++bad <= 10)
            std::cout << "\tidx " << i << " data " << C[i] << " gold " << G[i] << "\n";
    }
    std::cout << label << ": max abs diff " << abs_max << ", max rel diff " << rel_max << ", pass rate "
              << 100.0 * (double)(n - bad) / (double)n << "%\n";
    return bad == 0;
}

// The relative error this library is held to beside the reference's pass rule (which
// at these input scales admits almost any output through its absolute bound):
// max |C - G| / max(|G|, f * rms(G)), f = 1e-2 for DT outputs (tolerance 2e-3 fp16,
// 1e-2 bf16) and 0.25 for fp32 outputs (2e-4), as tests/helpers.py checks it.  Printed
// only; the pass/fail status stays the reference's.
inline void report_rel(const Epilogue &e, const unsigned char *C, const unsigned char *G, size_t n,
                       const std::string &label) {
    auto val = [&](const unsigned char *X, size_t i) -> double {
        if (e.out_f32) {
            float v;
            std::memcpy(&v, X + 4 * i, 4);
            return v;
        }
        uint16_t h;
        std::memcpy(&h, X + 2 * i, 2);
        return tof(h);
    };
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) ss += val(G, i) * val(G, i);
    const double floor = (e.out_f32 ? 0.25 : 1e-2) * std::sqrt(ss / (double)(n ? n : 1));
    double r = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double g = val(G, i), d = std::fabs(val(C, i) - g);
        const double q = d / std::max(std::max(std::fabs(g), floor), 1e-30);
        r = std::max(r, std::isnan(q) ? INFINITY : q);
    }
    const double tol = e.out_f32 ? 2e-4 : (bf16_mode() ? 1e-2 : 2e-3);
    std::cout << label << ": max rel err " << r << " (tolerance " << tol << ": " << (r <= tol ? "within" : "OVER")
              << ")\n";
}

inline bool compare_out(const Epilogue &e, const unsigned char *C, const unsigned char *G, size_t n,
                        const std::string &label) {
    report_rel(e, C, G, n, label);
    if (e.out_f32) return compare_f32((const float *)C, (const float *)G, n, label);
    return compare_dt((const uint16_t *)C, (const uint16_t *)G, n, label, e.abs_tol(), e.ulp_tol());
}

// ---- CUDA / library plumbing ---------------------------------------------------------------
inline void cuda_check(cudaError_t e, const char *what, int line) {
    if (e != cudaSuccess) {
        std::cerr << what << " failed: " << cudaGetErrorString(e) << " (line " << line << ")\n";
        std::exit(1);
    }
}
#define DRV_CUDA(x) ::drv::cuda_check((x), #x, __LINE__)

inline void lib_check(int st, const char *what, int line) {
    if (st != TERNOCL_OK) {
        std::cerr << what << " failed: " << ternocl_status_string(st) << " (" << ternocl_last_error() << ", line "
                  << line << ")\n";
        std::exit(1);
    }
}
#define DRV_LIB(x) ::drv::lib_check((x), #x, __LINE__)

// device copy of a host vector (nullptr for an empty one)
template <class T>
inline T *to_device(const std::vector<T> &h) {
    if (h.empty()) return nullptr;
    void *p = nullptr;
    DRV_CUDA(cudaMalloc(&p, h.size() * sizeof(T)));
    DRV_CUDA(cudaMemcpy(p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return (T *)p;
}
inline void *device_alloc(size_t bytes, int fill = 0) {
    void *p = nullptr;
    DRV_CUDA(cudaMalloc(&p, bytes ? bytes : 16));
    DRV_CUDA(cudaMemset(p, fill, bytes ? bytes : 16));
    return p;
}

inline std::string device_name() {
    int dev = 0;
    cudaDeviceProp prop;
    DRV_CUDA(cudaGetDevice(&dev));
    DRV_CUDA(cudaGetDeviceProperties(&prop, dev));
    return prop.name;
}

// Theoretical HBM bandwidth (GB/s) from the device attributes, for the roofline line.
inline double hbm_peak_gbs() {
    int dev = 0, clk_khz = 0, bus_bits = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0.0;
    cudaDeviceGetAttribute(&clk_khz, cudaDevAttrMemoryClockRate, dev);
    cudaDeviceGetAttribute(&bus_bits, cudaDevAttrGlobalMemoryBusWidth, dev);
    return 2.0 * clk_khz * 1e3 * (bus_bits / 8.0) / 1e9;
}

// One launch timed the reference drivers' way: blocking per launch, host time around
// launch + wait, device time between two events around the launch.  The reference reads
// the kernel's own start and end (OpenCL profiling info); to keep the host's launch cost
// out of the device time here, the stream is held by a host function until both events
// and the launch are queued, so the GPU runs them back to back.
struct LaunchTimer {
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    LaunchTimer() {
        DRV_CUDA(cudaEventCreate(&e0));
        DRV_CUDA(cudaEventCreate(&e1));
    }
    ~LaunchTimer() {
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    static void CUDART_CB hold(void *flag) {
        // released by the launching thread right after it has queued the launch
        const auto t0 = std::chrono::steady_clock::now();
        while (!__atomic_load_n((int *)flag, __ATOMIC_ACQUIRE))
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) break;
    }
    template <class F>
    void run(F &&launch, double &dev_ms, double &host_ms) {
        int flag = 0;
        DRV_CUDA(cudaLaunchHostFunc(0, hold, &flag));
        DRV_CUDA(cudaEventRecord(e0, 0));
        const auto t0 = std::chrono::high_resolution_clock::now();
        launch();
        DRV_CUDA(cudaEventRecord(e1, 0));
        __atomic_store_n(&flag, 1, __ATOMIC_RELEASE);
        DRV_CUDA(cudaEventSynchronize(e1));
        const auto t1 = std::chrono::high_resolution_clock::now();
        float ms = 0.0f;
        DRV_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        dev_ms = ms;
        host_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    }
};

inline void check_device_error() {
    const int e = ternocl_device_error(1);
    if (e > 0) std::cout << "device error word: 0x" << std::hex << e << std::dec << "\n";
}

// ---- flags ----------------------------------------------------------------------------
// The reference's tile and Xe2 code-generation flags select OpenCL -D options there; the
// CUDA kernels pick their own launch shapes, so these are accepted and reported.
struct Flags {
    int argc;
    char **argv;
    int i = 1;
    std::vector<std::string> ignored;
    bool is(const char *name) const { return std::strcmp(argv[i], name) == 0; }
    bool has_value() const { return i + 1 < argc; }
    const char *value() { return argv[++i]; }
    int ival() { return std::atoi(value()); }
    double fval() { return std::atof(value()); }
    void ignore(bool takes_value) {
        std::string s = argv[i];
        if (takes_value && has_value()) s += std::string(" ") + value();
        ignored.push_back(s);
    }
};

inline void report_ignored(const Flags &f) {
    if (f.ignored.empty()) return;
    std::cout << "Ignored (OpenCL/Xe2 tuning, the CUDA kernels choose their own launch shapes):";
    for (const auto &s : f.ignored) std::cout << " " << s;
    std::cout << "\n";
}

// --dtype: returns false on a bad value
inline bool parse_dtype(Flags &f) {
    const std::string d = f.value();
    if (d != "fp16" && d != "bf16") return false;
    bf16_mode() = d == "bf16";
    return true;
}

}  // namespace drv
