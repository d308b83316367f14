// Command-line driver of the BITCOS upconvert GEMV/GEMM, with the flags and stdout lines
// of bitcos_fp16_upcvt/main.cpp (:337-387): random ternary weights at zero density --z
// packed by libternocl's host packer (bit-identical to the reference's bitcos_random for
// the same seed), slice ranks for --ls K-slices, the fp32 gold from the decoded columns,
// rotation over distinct weight sets, the actual-bytes and int2-equivalent GiB/s.
// Kernel: the M-tiled tcgen05 GEMM when M >= 64 or --mt-m is given, else the GEMV
// (the reference selects its M-tiled kernel only with --mt-m).
#include "driver_common.hpp"

using namespace drv;

namespace {

struct Config {
    int m = 1, n = 4096, k = 4096, iters = 50;
    double z = 0.40;
    bool validate = true, distinct_sets = false;
    int num_sets = 0, ls = 0;
    double weights_gib = 2.0;
    bool mt_forced = false;
    Epilogue epi;
};

struct Bitcos {
    std::vector<uint32_t> buf;
    int K = 0, N = 0;
    size_t bytes() const { return buf.size() * 4; }
    // codes of column n in row order (bitmap | offsets | signs, 1 -> -1)
    void decode_col(int n, int8_t *out) const {
        const uint32_t *bm = buf.data();
        const uint32_t *off = bm + (size_t)(K / 32) * N;
        const uint32_t *sg = off + N + off[n];
        uint32_t rank = 0;
        for (int k = 0; k < K; ++k) {
            if (!((bm[(size_t)(k / 32) * N + n] >> (k % 32)) & 1u)) {
                out[k] = 0;
                continue;
            }
            out[k] = ((sg[rank >> 5] >> (rank & 31)) & 1u) ? -1 : 1;
            ++rank;
        }
    }
    double zero_density() const {
        size_t nz = 0;
        for (size_t i = 0; i < (size_t)(K / 32) * N; ++i) nz += (size_t)__builtin_popcount(buf[i]);
        return 1.0 - (double)nz / ((double)K * N);
    }
};

Bitcos make_bitcos(int K, int N, double z, uint64_t seed) {
    Bitcos b;
    b.K = K;
    b.N = N;
    const size_t n = ternocl_bitcos_random(K, N, z, seed, nullptr, 0);
    b.buf.resize(n);
    ternocl_bitcos_random(K, N, z, seed, b.buf.data(), n);
    return b;
}

void host_gold(const std::vector<uint16_t> &A, const Bitcos &b, const std::vector<uint16_t> &S, std::vector<float> &acc,
               int M) {
    const int K = b.K, N = b.N;
    acc.assign((size_t)M * N, 0.0f);
#pragma omp parallel
    {
        std::vector<int8_t> codes(K);
#pragma omp for schedule(dynamic, 16)
        for (int n = 0; n < N; ++n) {
            b.decode_col(n, codes.data());
            for (int m = 0; m < M; ++m) {
                float a = 0.0f;
                for (int g = 0; g < K / kGS; ++g) {
                    float part = 0.0f;
                    for (int p = 0; p < kGS; ++p) {
                        const int k = g * kGS + p;
                        if (codes[k]) part += tof(A[(size_t)m * K + k]) * (float)codes[k];
                    }
                    a += part * tof(S[(size_t)g * N + n]);
                }
                acc[(size_t)m * N + n] = a;
            }
        }
    }
}

void usage(const char *prog) {
    std::cout << "Usage: " << prog
              << " [--m M] [--n N] [--k K] [--z Z] [--dtype fp16|bf16] [--iters N] [--no-validate]\n"
                 "       [--distinct-sets] [--sets N | --weights-gib G] [--ls L] [--seed S] [--postop 0|1|2|3|4]\n"
                 "       [--out-f32] [--mt-m M] (selects the M-tiled GEMM at any M)\n"
                 "       accepted and ignored: --sgm --nsg --wgn --mt-n --wg-m --wg-n --int-apply --simt-mul\n"
                 "       --cl --opts --build-log\n";
}

int run(Config cfg, const Flags &flags) {
    const int M = cfg.m, N = cfg.n, K = cfg.k;
    if (cfg.ls == 0) cfg.ls = 4;
    while (cfg.ls > 1 && K % (64 * cfg.ls)) cfg.ls /= 2;
    if (M < 1 || N < 16 || K < kGS || K % kGS || N % 16 || K % (64 * cfg.ls)) {
        std::cerr << "need K % 128 == 0, N % 16 == 0 and K % (64 * LS) == 0\n";
        return 1;
    }
    const bool mt = cfg.mt_forced || M >= 64;
    const Epilogue &ep = cfg.epi;
    std::cout << "Device: " << device_name() << "\n"
              << "Problem: M=" << M << " N=" << N << " K=" << K << " scale_gs=" << kGS << " z=" << cfg.z
              << " dtype=" << dt_name() << " epilogue=" << ep.name() << "\n"
              << "Kernel: " << (mt ? "tcgen05 GEMM (sm_100a)" : "decode GEMV (sm_100a)") << " ls=" << cfg.ls
              << ", libternocl " << ternocl_version() << "\n";
    report_ignored(flags);

    const size_t os = ep.out_size();
    const size_t size_a = (size_t)M * K, size_c = (size_t)M * N, size_s = (size_t)(K / kGS) * N;
    std::vector<uint16_t> A(size_a), S(size_s), Oth;
    std::vector<unsigned char> Bias, Ch(size_c * os);
    std::vector<uint32_t> SR;
    Bitcos B;
    uint64_t seed = seed_fixed() ? seed_base() : (((uint64_t)std::random_device{}() << 32) ^ std::random_device{}());
    auto fill = [&] {
#pragma omp parallel for
        for (long long i = 0; i < (long long)size_a; ++i) A[i] = fromf(rnd_uniform(-5.0f, 5.0f));
        for (auto &s : S) s = fromf(rnd_uniform(0.0f, 15.0f) + 0.75f);
        B = make_bitcos(K, N, cfg.z, seed++);
        SR.assign(cfg.ls > 1 ? (size_t)(cfg.ls - 1) * N : 1, 0u);
        if (cfg.ls > 1) DRV_LIB(ternocl_bitcos_slice_ranks(B.buf.data(), K, N, cfg.ls, SR.data()));
        fill_epilogue_inputs(ep, Oth, Bias, M, N);
    };
    fill();
    const double wbytes_set = (double)B.bytes() + size_s * 2.0;
    const int sets = cfg.num_sets > 0 ? cfg.num_sets
                                      : std::max(1, (int)std::ceil(cfg.weights_gib * (1 << 30) / wbytes_set));
    std::cout << "BITCOS: measured z " << std::setprecision(4) << B.zero_density() << ", "
              << 8.0 * B.bytes() / ((double)K * N) << " bits/weight (+scales); weights " << wbytes_set / (1 << 20)
              << " MiB/set, " << sets << " distinct sets -> " << std::fixed << std::setprecision(3)
              << wbytes_set * sets / (1 << 30) << " GiB\n";
    std::cout.unsetf(std::ios::floatfield);
    std::cout << std::setprecision(6);

    const int ngold = cfg.validate ? (cfg.distinct_sets ? sets : 1) : 0;
    std::vector<std::vector<unsigned char>> gold(ngold);
    std::vector<float> acc;
    auto make_gold = [&](std::vector<unsigned char> &g) {
        host_gold(A, B, S, acc, M);
        g.resize(size_c * os);
        apply_epilogue(ep, acc.data(), Oth.data(), Bias.data(), g.data(), M, N);
    };
    if (cfg.validate) make_gold(gold[0]);

    struct Set {
        uint16_t *A, *S, *O;
        uint32_t *B, *SR;
        void *C, *Bias;
        size_t bbytes;
    };
    std::vector<Set> dev(sets);
    for (int s = 0; s < sets; ++s) {
        if (cfg.distinct_sets && s > 0) {
            fill();
            if (cfg.validate) make_gold(gold[s]);
        }
        dev[s].A = to_device(A);
        dev[s].B = to_device(B.buf);
        dev[s].bbytes = B.bytes();
        dev[s].SR = to_device(SR);
        dev[s].S = to_device(S);
        dev[s].O = to_device(Oth);
        dev[s].Bias = to_device(Bias);
        dev[s].C = device_alloc(size_c * os);
    }
    const int algo = mt ? TERNOCL_ALGO_GEMM : TERNOCL_ALGO_GEMV;
    DRV_CUDA(cudaDeviceSynchronize());

    LaunchTimer timer;
    double dev_ms = 0.0, host_ms = 0.0, bsum = 0.0;
    int timed = 0;
    for (int it = 0; it < sets + cfg.iters; ++it) {
        const Set &d = dev[it % sets];
        double dms = 0.0, hms = 0.0;
        timer.run(
            [&] {
                DRV_LIB(ternocl_bitcos_upcvt(d.A, d.B, d.S, cfg.ls > 1 ? d.SR : nullptr, cfg.ls, d.C, d.O, d.Bias, M,
                                             N, K, dt_code(), ep.postop, ep.out_f32, algo, nullptr));
            },
            dms, hms);
        if (it >= sets) {
            dev_ms += dms;
            host_ms += hms;
            bsum += (double)d.bbytes;
            ++timed;
        }
    }
    if (timed) {
        const double dms = dev_ms / timed, hms = host_ms / timed;
        // actual bytes: A + BITCOS buffer + scales + C (+ epilogue operands)
        const double bytes = (double)M * K * 2 + bsum / timed + (double)(K / kGS) * N * 2 + (double)M * N * os +
                             (ep.needs_other() ? (double)M * N * 2 : 0.0) + (ep.needs_bias() ? (double)N * os : 0.0);
        // the same weight count at 2 bits per weight
        const double bytes_i2 = bytes - bsum / timed + (double)K * N / 4.0;
        const double gib = 1024.0 * 1024.0 * 1024.0, flop = 2.0 * M * N * K;
        std::cout << std::fixed << std::setprecision(5) << "Avg host  time: " << hms << " ms ("
                  << flop / (hms * 1e-3) / 1e9 << " GFLOPS)\n"
                  << "Avg dev   time: " << dms << " ms (" << flop / (dms * 1e-3) / 1e9 << " GFLOPS, "
                  << bytes / (dms * 1e-3) / gib << " GiB/s, int2-equiv " << bytes_i2 / (dms * 1e-3) / gib << " GiB/s)\n"
                  << "Bytes/GEMM: " << bytes / (1 << 20) << " MiB\n";
        const double peak = hbm_peak_gbs();
        std::cout << "Roofline: " << bytes / (dms * 1e-3) / 1e9 << " GB/s of " << peak << " GB/s HBM (theoretical, "
                  << 100.0 * bytes / (dms * 1e-3) / 1e9 / std::max(peak, 1e-9) << "%), " << flop / (dms * 1e-3) / 1e12
                  << " TFLOPS\n";
        std::cout.unsetf(std::ios::floatfield);
        std::cout << std::setprecision(6);
    }
    check_device_error();

    if (cfg.validate) {
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
        cudaFree(d.SR);
        cudaFree(d.S);
        cudaFree(d.O);
        cudaFree(d.Bias);
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
        else if (f.is("--z") && v) cfg.z = f.fval();
        else if (f.is("--dtype") && v) {
            if (!parse_dtype(f)) {
                std::cerr << "--dtype fp16|bf16\n";
                return 1;
            }
        } else if (f.is("--iters") && v) cfg.iters = f.ival();
        else if (f.is("--sets") && v) cfg.num_sets = f.ival();
        else if (f.is("--weights-gib") && v) cfg.weights_gib = f.fval();
        else if (f.is("--seed") && v) seed_base() = (uint64_t)std::strtoull(f.value(), nullptr, 10), seed_fixed() = true;
        else if (f.is("--no-validate")) cfg.validate = false;
        else if (f.is("--distinct-sets")) cfg.distinct_sets = true;
        else if (f.is("--ls") && v) cfg.ls = f.ival();
        else if (f.is("--postop") && v) {
            cfg.epi.postop = f.ival();
            if (cfg.epi.postop < 0 || cfg.epi.postop > 4) {
                std::cerr << "--postop 0..4\n";
                return 1;
            }
        } else if (f.is("--out-f32")) cfg.epi.out_f32 = true;
        else if (f.is("--mt-m") && v) {
            cfg.mt_forced = f.ival() > 0;
            f.ignored.push_back("--mt-m tile size");
        } else if ((f.is("--sgm") || f.is("--nsg") || f.is("--wgn") || f.is("--mt-n") || f.is("--wg-m") ||
                    f.is("--wg-n") || f.is("--cl") || f.is("--opts")) &&
                   v)
            f.ignore(true);
        else if (f.is("--int-apply") || f.is("--simt-mul") || f.is("--build-log")) f.ignore(false);
        else {
            usage(argv[0]);
            return f.is("-h") || f.is("--help") ? 0 : 1;
        }
    }
    return run(cfg, f);
}
