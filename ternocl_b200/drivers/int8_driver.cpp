// Command-line driver of the s8 x s2 path (activation quantisation pre-kernel + int8 x
// int2 GEMV/GEMM), with the flags and stdout lines of int2_via_int2_x_int8_dpas/main.cpp
// (:440-488): the A fill is fake-quantised (A = DT(q / SA) with q on the int8 grid,
// optionally --offgrid LSB off it) so the per-group scales are exact, the host gold
// quantises with round-to-nearest-even and accumulates int32 dots per 128-group,
// the pre-kernel and the GEMM are timed separately ("Avg dev   pre :", "Avg dev   gemm:")
// and the device scales of the last set are checked bit for bit against the host's.
#include <cfloat>

#include "driver_common.hpp"

using namespace drv;

namespace {

struct Config {
    int m = 1, n = 4096, k = 4096, iters = 50;
    int qmode = 1;  // 0: int8 A written by the pre-kernel; 1: A quantised inside the GEMM
    bool validate = true, distinct_sets = false;
    int num_sets = 0;
    double weights_gib = 2.0;
    bool mt_forced = false;
    float offgrid = 0.0f;
    Epilogue epi;
};

inline int ldsa(int M) { return (M + 31) & ~31; }

// SA[g, m] = DT(127 / max(FLT_EPSILON, max |A[m, group g]|))
void host_scales(const std::vector<uint16_t> &A, std::vector<uint16_t> &SA, int M, int K) {
#pragma omp parallel for
    for (int m = 0; m < M; ++m)
        for (int g = 0; g < K / kGS; ++g) {
            float mx = FLT_EPSILON;
            for (int p = 0; p < kGS; ++p) mx = std::max(mx, std::fabs(tof(A[(size_t)m * K + g * kGS + p])));
            SA[(size_t)g * ldsa(M) + m] = fromf(127.0f / mx);
        }
}

inline int8_t quant(float a, float sa) {
    const long v = std::lrintf(a * sa);  // round to nearest even
    return (int8_t)std::min(127L, std::max(-128L, v));
}

void host_gold(const std::vector<uint16_t> &A, const std::vector<uint32_t> &B, const std::vector<uint16_t> &SA,
               const std::vector<uint16_t> &SB, std::vector<float> &acc, int M, int K, int N) {
    std::vector<int8_t> q((size_t)M * K);
#pragma omp parallel for
    for (int m = 0; m < M; ++m)
        for (int k = 0; k < K; ++k)
            q[(size_t)m * K + k] = quant(tof(A[(size_t)m * K + k]), tof(SA[(size_t)(k / kGS) * ldsa(M) + m]));
    acc.assign((size_t)M * N, 0.0f);
#pragma omp parallel
    {
        int8_t w[kGS];
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n)
            for (int g = 0; g < K / kGS; ++g) {
                for (int p = 0; p < kGS; ++p) {
                    const int k = g * kGS + p;
                    w[p] = (int8_t)int2_code_value((B[(size_t)(k / 16) * N + n] >> (2 * (k % 16))) & 3u);
                }
                const float sb = tof(SB[(size_t)g * N + n]);
                for (int m = 0; m < M; ++m) {
                    int32_t dot = 0;
                    const int8_t *qr = &q[(size_t)m * K + (size_t)g * kGS];
                    for (int p = 0; p < kGS; ++p) dot += (int32_t)qr[p] * w[p];
                    const float sa = tof(SA[(size_t)g * ldsa(M) + m]);
                    const float inv = sa == 0.0f ? 0.0f : 1.0f / sa;
                    acc[(size_t)m * N + n] += (float)dot * (sb * inv);
                }
            }
    }
}

void usage(const char *prog) {
    std::cout << "Usage: " << prog
              << " [--m M] [--n N] [--k K] [--dtype fp16|bf16] [--qmode 0|1] [--iters N] [--no-validate]\n"
                 "       [--distinct-sets] [--sets N | --weights-gib G] [--offgrid F] [--seed S]\n"
                 "       [--postop 0|1|2|3|4] [--out-f32] [--mt-m M] (selects the M-tiled GEMM at any M)\n"
                 "       accepted and ignored: --sgm --nsg --wgn --ls --u --mt-n --wg-m --wg-n --cl --opts --build-log\n"
                 "       epilogue: 0 none, 1 silu(acc)*other, 2 acc+other, 3 acc+bias[n], 4 sigmoid(acc);\n"
                 "       --out-f32 = fp32 C/bias\n"
                 "qmode: 0 upfront int8 A, 1 quantize A in the GEMM\n";
}

int run(const Config &cfg, const Flags &flags) {
    const int M = cfg.m, N = cfg.n, K = cfg.k;
    if (M < 1 || N < 16 || K < kGS || K % kGS || N % 16) {
        std::cerr << "need K % 128 == 0 and N % 16 == 0\n";
        return 1;
    }
    if (cfg.qmode < 0 || cfg.qmode > 1) {
        std::cerr << "--qmode 0|1\n";
        return 1;
    }
    const bool mt = cfg.mt_forced || M >= 64;
    const Epilogue &ep = cfg.epi;
    static const char *qname[] = {"upfront (int8 A + scale pre-kernel)", "scale pre-kernel, quantize in the GEMM"};
    std::cout << "Device: " << device_name() << "\n"
              << "Problem: M=" << M << " N=" << N << " K=" << K << " scale_gs=" << kGS << " dtype=" << dt_name()
              << " epilogue=" << ep.name() << "\n"
              << "A quant: qmode=" << cfg.qmode << " " << qname[cfg.qmode] << "\n"
              << "Kernel: "
              << (mt && cfg.qmode == 0 ? "tcgen05 kind::i8 GEMM (sm_100a)" : "s8 x s2 decode GEMV (sm_100a)")
              << ", libternocl " << ternocl_version() << "\n";
    report_ignored(flags);

    const size_t size_a = (size_t)M * K, size_b = (size_t)(K / 16) * N;
    const size_t size_c = (size_t)M * N, size_sb = (size_t)(K / kGS) * N;
    const size_t size_sa = (size_t)(K / kGS) * ldsa(M);
    const size_t os = ep.out_size();
    const double bytes_set = size_a * 3.0 + size_b * 4.0 + size_c * (double)os + (size_sb + size_sa) * 2.0 +
                             (ep.needs_other() ? size_c * 2.0 : 0.0) + (ep.needs_bias() ? N * (double)os : 0.0);
    const double wbytes_set = size_b * 4.0 + size_sb * 2.0;
    const int sets = cfg.num_sets > 0 ? cfg.num_sets
                                      : std::max(1, (int)std::ceil(cfg.weights_gib * (1 << 30) / wbytes_set));
    std::cout << "Per-set bytes: " << bytes_set / (1 << 20) << " MiB (weights " << wbytes_set / (1 << 20)
              << " MiB); using " << sets << " distinct sets -> weights " << std::fixed << std::setprecision(3)
              << wbytes_set * sets / (1 << 30) << " GiB, total " << bytes_set * sets / (1 << 30) << " GiB\n";
    std::cout.unsetf(std::ios::floatfield);
    std::cout << std::setprecision(6);

    std::vector<uint16_t> A(size_a), SA(size_sa, 0), SB(size_sb), Oth;
    std::vector<unsigned char> Bias, Ch(size_c * os);
    std::vector<uint32_t> B(size_b);
    auto fill = [&] {
#pragma omp parallel for
        for (long long i = 0; i < (long long)size_a; ++i) A[i] = fromf(rnd_uniform(-5.0f, 5.0f));
#pragma omp parallel for
        for (long long i = 0; i < (long long)size_b; ++i) B[i] = rnd_int2_word();
        for (auto &s : SB) s = fromf(rnd_uniform(0.0f, 15.0f) + 0.75f);
        // fake-quantise A onto the int8 grid of its own scales (+- offgrid LSB), then
        // take the scales of the result
        host_scales(A, SA, M, K);
#pragma omp parallel for
        for (int m = 0; m < M; ++m)
            for (int k = 0; k < K; ++k) {
                const float sa = tof(SA[(size_t)(k / kGS) * ldsa(M) + m]);
                const int q = quant(tof(A[(size_t)m * K + k]), sa);
                const float off = q >= 0 ? cfg.offgrid : -cfg.offgrid;
                A[(size_t)m * K + k] = fromf(((float)q + off) * (1.0f / sa));
            }
        host_scales(A, SA, M, K);
        fill_epilogue_inputs(ep, Oth, Bias, M, N);
    };
    fill();

    const int ngold = cfg.validate ? (cfg.distinct_sets ? sets : 1) : 0;
    std::vector<std::vector<unsigned char>> gold(ngold);
    std::vector<float> acc;
    auto make_gold = [&](std::vector<unsigned char> &g) {
        host_gold(A, B, SA, SB, acc, M, K, N);
        g.resize(size_c * os);
        apply_epilogue(ep, acc.data(), Oth.data(), Bias.data(), g.data(), M, N);
    };
    if (cfg.validate) make_gold(gold[0]);

    struct Set {
        uint16_t *A, *SB, *O;
        uint32_t *B;
        void *SA, *C, *Bias;
        int8_t *Aq;
    };
    std::vector<Set> dev(sets);
    for (int s = 0; s < sets; ++s) {
        if (cfg.distinct_sets && s > 0) {
            fill();
            if (cfg.validate) make_gold(gold[s]);
        }
        dev[s].A = to_device(A);
        dev[s].B = to_device(B);
        dev[s].SB = to_device(SB);
        dev[s].O = to_device(Oth);
        dev[s].Bias = to_device(Bias);
        // SA and Aq are device outputs: filled with junk so that a missing write fails
        dev[s].SA = device_alloc(size_sa * 2, 0x5a);
        dev[s].Aq = cfg.qmode == 0 ? (int8_t *)device_alloc(size_a, 0x5a) : nullptr;
        dev[s].C = device_alloc(size_c * os);
    }
    const int algo = mt ? TERNOCL_ALGO_GEMM : TERNOCL_ALGO_GEMV;
    DRV_CUDA(cudaDeviceSynchronize());

    cudaEvent_t ev[3];
    for (auto &e : ev) DRV_CUDA(cudaEventCreate(&e));
    double pre_ms = 0.0, gemm_ms = 0.0, host_ms = 0.0;
    int timed = 0;
    for (int it = 0; it < sets + cfg.iters; ++it) {
        const Set &d = dev[it % sets];
        int flag = 0;  // holds the stream until both launches are queued (LaunchTimer)
        DRV_CUDA(cudaLaunchHostFunc(0, LaunchTimer::hold, &flag));
        DRV_CUDA(cudaEventRecord(ev[0], 0));
        const auto t0 = std::chrono::high_resolution_clock::now();
        DRV_LIB(ternocl_int8_quant_a(d.A, d.SA, d.Aq, M, K, dt_code(), nullptr));
        DRV_CUDA(cudaEventRecord(ev[1], 0));
        DRV_LIB(ternocl_int2_int8(d.A, d.Aq, d.SA, d.B, d.SB, d.C, d.O, d.Bias, M, N, K, dt_code(), ep.postop,
                                  ep.out_f32, cfg.qmode, algo, nullptr));
        DRV_CUDA(cudaEventRecord(ev[2], 0));
        __atomic_store_n(&flag, 1, __ATOMIC_RELEASE);
        DRV_CUDA(cudaEventSynchronize(ev[2]));
        const auto t1 = std::chrono::high_resolution_clock::now();
        if (it >= sets) {
            float a = 0.0f, b = 0.0f;
            DRV_CUDA(cudaEventElapsedTime(&a, ev[0], ev[1]));
            DRV_CUDA(cudaEventElapsedTime(&b, ev[1], ev[2]));
            pre_ms += a;
            gemm_ms += b;
            host_ms += std::chrono::duration<double, std::milli>(t1 - t0).count();
            ++timed;
        }
    }
    for (auto &e : ev) cudaEventDestroy(e);
    if (timed) {
        const double gms = gemm_ms / timed, pms = pre_ms / timed, hms = host_ms / timed, tms = gms + pms;
        // the upconvert driver's byte model (A DT + B + C + both scales)
        const double bytes = (double)M * K * 2 + (double)K * N / 4.0 + (double)M * N * os +
                             (double)(K / kGS) * (N + M) * 2 + (ep.needs_other() ? (double)M * N * 2 : 0.0) +
                             (ep.needs_bias() ? (double)N * os : 0.0);
        const double gib = 1024.0 * 1024.0 * 1024.0, flop = 2.0 * M * N * K;
        std::cout << std::fixed << std::setprecision(5) << "Avg host  time: " << hms << " ms ("
                  << flop / (hms * 1e-3) / 1e9 << " GFLOPS)\n"
                  << "Avg dev   pre : " << pms << " ms\n"
                  << "Avg dev   gemm: " << gms << " ms (" << flop / (gms * 1e-3) / 1e9 << " GFLOPS, "
                  << bytes / (gms * 1e-3) / gib << " GiB/s)\n"
                  << "Avg dev   time: " << tms << " ms (" << flop / (tms * 1e-3) / 1e9 << " GFLOPS, "
                  << bytes / (tms * 1e-3) / gib << " GiB/s)\n"
                  << "Bytes/GEMM: " << bytes / (1 << 20) << " MiB\n";
        const double peak = hbm_peak_gbs();
        std::cout << "Roofline: " << bytes / (tms * 1e-3) / 1e9 << " GB/s of " << peak << " GB/s HBM (theoretical, "
                  << 100.0 * bytes / (tms * 1e-3) / 1e9 / std::max(peak, 1e-9) << "%), " << flop / (tms * 1e-3) / 1e12
                  << " TOPS\n";
        std::cout.unsetf(std::ios::floatfield);
        std::cout << std::setprecision(6);
    }
    check_device_error();

    if (cfg.validate) {
        {  // device scales of the last set vs the host's (the last filled)
            std::vector<uint16_t> SAh(size_sa);
            DRV_CUDA(cudaMemcpy(SAh.data(), dev[sets - 1].SA, size_sa * 2, cudaMemcpyDeviceToHost));
            size_t diff = 0;
            for (int g = 0; g < K / kGS; ++g)
                for (int m = 0; m < M; ++m) {
                    const size_t i = (size_t)g * ldsa(M) + m;
                    diff += SAh[i] != SA[i];
                }
            std::cout << "scale_a: " << diff << "/" << (size_t)(K / kGS) * M << " differ from host\n";
        }
        int passed = 0;
        std::vector<unsigned char> C0;
        for (int s = 0; s < sets; ++s) {
            DRV_CUDA(cudaMemcpy(Ch.data(), dev[s].C, size_c * os, cudaMemcpyDeviceToHost));
            const auto &g = gold[cfg.distinct_sets ? s : 0];
            const std::string label = "validation [set " + std::to_string(s) + "/" + std::to_string(sets) + "]";
            bool ok;
            if (!cfg.distinct_sets && s > 0 && std::memcmp(Ch.data(), C0.data(), size_c * os) == 0) ok = true;
            else ok = compare_out(ep, Ch.data(), g.data(), size_c, label);
            if (s == 0) C0 = Ch;
            passed += ok;
            if (!ok) std::cout << "FAILED at set " << s << "\n";
            if (!cfg.distinct_sets && s == 0 && !ok) break;
        }
        std::cout << "Validation summary: " << passed << "/" << sets << " sets PASSED\n";
    }
    for (auto &d : dev) {
        cudaFree(d.A);
        cudaFree(d.B);
        cudaFree(d.SB);
        cudaFree(d.O);
        cudaFree(d.Bias);
        cudaFree(d.SA);
        cudaFree(d.Aq);
        cudaFree(d.C);
    }
    return 0;
}

}  // namespace

int main(int argc, char **argv) {
    Config cfg;
    Flags f{argc, argv};
    for (; f.i < argc; ++f.i) {
        const bool v = f.has_value();
        if (f.is("--m") && v) cfg.m = f.ival();
        else if (f.is("--n") && v) cfg.n = f.ival();
        else if (f.is("--k") && v) cfg.k = f.ival();
        else if (f.is("--dtype") && v) {
            if (!parse_dtype(f)) {
                std::cerr << "--dtype fp16|bf16\n";
                return 1;
            }
        } else if (f.is("--qmode") && v) cfg.qmode = f.ival();
        else if (f.is("--postop") && v) {
            cfg.epi.postop = f.ival();
            if (cfg.epi.postop < 0 || cfg.epi.postop > 4) {
                std::cerr << "--postop 0..4\n";
                return 1;
            }
        } else if (f.is("--out-f32")) cfg.epi.out_f32 = true;
        else if (f.is("--iters") && v) cfg.iters = f.ival();
        else if (f.is("--sets") && v) cfg.num_sets = f.ival();
        else if (f.is("--weights-gib") && v) cfg.weights_gib = f.fval();
        else if (f.is("--seed") && v) seed_base() = (uint64_t)std::strtoull(f.value(), nullptr, 10), seed_fixed() = true;
        else if (f.is("--no-validate")) cfg.validate = false;
        else if (f.is("--distinct-sets")) cfg.distinct_sets = true;
        else if (f.is("--offgrid") && v) cfg.offgrid = (float)f.fval();
        else if (f.is("--mt-m") && v) {
            cfg.mt_forced = f.ival() > 0;
            f.ignored.push_back("--mt-m tile size");
        } else if ((f.is("--sgm") || f.is("--nsg") || f.is("--wgn") || f.is("--ls") || f.is("--u") ||
                    f.is("--mt-n") || f.is("--wg-m") || f.is("--wg-n") || f.is("--cl") || f.is("--opts")) &&
                   v)
            f.ignore(true);
        else if (f.is("--build-log")) f.ignore(false);
        else {
            usage(argv[0]);
            return f.is("-h") || f.is("--help") ? 0 : 1;
        }
    }
    return run(cfg, f);
}
