// Command-line driver of the int2 MoE decode layer, with the flags and stdout lines of
// int2_moe/main.cpp (:91-336): T tokens routed to TOPK distinct experts of E (uniform
// permutation per token, gate weights U(0.05, 1) normalised), --sets layers of gate / up /
// down weights at distinct addresses (the same values unless --distinct), the double-
// precision check of the layer output ("check: ... PASS|FAIL", main.cpp:267-291) and per-
// kernel median device times over the layers (gate_up, down and reduce, or gate_up and
// down_sum with --fused) with the bytes of the experts actually touched.
#include <numeric>

#include "driver_common.hpp"

using namespace drv;

namespace {

struct Proj {
    int E, K, N;
    std::vector<uint32_t> B;  // [E, K/16, N]
    std::vector<uint16_t> S;  // [E, K/128, N]
    uint32_t *dB = nullptr;
    uint16_t *dS = nullptr;
    size_t b_words() const { return (size_t)E * (K / 16) * N; }
    size_t s_elems() const { return (size_t)E * (K / kGS) * N; }
    double w(int e, int k, int n) const {
        const uint32_t word = B[((size_t)e * (K / 16) + k / 16) * N + n];
        return (double)int2_code_value((word >> (2 * (k % 16))) & 3u) *
               tof(S[((size_t)e * (K / kGS) + k / kGS) * N + n]);
    }
};

void fill_proj(Proj &p) {
    p.B.resize(p.b_words());
    p.S.resize(p.s_elems());
#pragma omp parallel for
    for (long long i = 0; i < (long long)p.B.size(); ++i) p.B[i] = rnd_int2_word();
    for (auto &s : p.S) s = fromf(rnd_uniform(0.005f, 0.05f));
}

}  // namespace

int main(int argc, char **argv) {
    int T = 1, E = 128, TOPK = 8, H = 2048, I = 768, sets = 48, iters = 20;
    bool fused = false, distinct = false;
    Flags f{argc, argv};
    for (; f.i < argc; ++f.i) {
        const bool v = f.has_value();
        if (f.is("--t") && v) T = f.ival();
        else if (f.is("--e") && v) E = f.ival();
        else if (f.is("--topk") && v) TOPK = f.ival();
        else if (f.is("--h") && v) H = f.ival();
        else if (f.is("--i") && v) I = f.ival();
        else if (f.is("--sets") && v) sets = f.ival();
        else if (f.is("--iters") && v) iters = f.ival();
        else if (f.is("--fused")) fused = true;
        else if (f.is("--distinct")) distinct = true;
        else if (f.is("--seed") && v) seed_base() = (uint64_t)std::strtoull(f.value(), nullptr, 10), seed_fixed() = true;
        else if (f.is("--dtype") && v) {
            if (!parse_dtype(f)) {
                std::cerr << "--dtype fp16|bf16\n";
                return 1;
            }
        } else if ((f.is("--gu") || f.is("--dn") || f.is("--dir")) && v) f.ignore(true);
        else {
            std::cerr << "usage: " << argv[0]
                      << " [--t T] [--e E] [--topk K] [--h H] [--i I] [--sets S] [--iters N] [--fused] [--distinct]"
                         " [--dtype fp16|bf16] [--seed S]  (accepted and ignored: --gu --dn --dir)\n";
            return 1;
        }
    }
    if (T < 1 || E < 1 || TOPK < 1 || TOPK > E || H % kGS || I % kGS || sets < 1 || iters < 1) {
        std::cerr << "need 1 <= topk <= E, H and I multiples of 128\n";
        return 1;
    }
    if (!seed_fixed()) seed_base() = 42, seed_fixed() = true;  // the reference seeds its layer with 42
    const int G = T * TOPK, dt = dt_code();
    std::cout << "Device: " << device_name() << "\nProblem: T=" << T << " E=" << E << " topk=" << TOPK << " H=" << H
              << " I=" << I << " sets=" << sets << " dtype=" << dt_name()
              << "\nKernels: integer-MMA decode GEMVs (sm_100a), " << (fused ? "gate_up + down_sum" : "gate_up + down + reduce")
              << "\n";
    report_ignored(f);

    std::vector<Proj> gate(sets, Proj{E, H, I}), up(sets, Proj{E, H, I}), down(sets, Proj{E, I, H});
    for (int l = 0; l < sets; ++l)
        for (auto *pp : {&gate, &up, &down}) {
            Proj &p = (*pp)[l];
            if (l == 0 || distinct) fill_proj(p);
            const Proj &src = distinct ? p : (*pp)[0];
            p.dB = to_device(src.B);
            p.dS = to_device(src.S);
            if (l > 0 && distinct) {
                std::vector<uint32_t>().swap(p.B);
                std::vector<uint16_t>().swap(p.S);
            }
        }

    std::vector<uint16_t> X((size_t)T * H), RW(G);
    std::vector<int32_t> ids(G);
    for (auto &x : X) x = fromf(rnd_uniform(-1.0f, 1.0f));
    for (int t = 0; t < T; ++t) {
        std::vector<int> perm(E);
        std::iota(perm.begin(), perm.end(), 0);
        for (int k = E - 1; k > 0; --k) std::swap(perm[k], perm[rnd_u32() % (uint32_t)(k + 1)]);
        float sum = 0.0f;
        std::vector<float> w(TOPK);
        for (int j = 0; j < TOPK; ++j) sum += (w[j] = rnd_uniform(0.05f, 1.0f));
        for (int j = 0; j < TOPK; ++j) {
            ids[(size_t)t * TOPK + j] = perm[j];
            RW[(size_t)t * TOPK + j] = fromf(w[j] / sum);
        }
    }
    uint16_t *dX = to_device(X), *dRW = to_device(RW);
    int32_t *dIds = to_device(ids);
    void *dH = device_alloc((size_t)G * I * 2), *dO = device_alloc((size_t)T * H * 2);
    float *dY = (float *)device_alloc((size_t)G * H * 4);

    cudaEvent_t ev[4];
    for (auto &e : ev) DRV_CUDA(cudaEventCreate(&e));
    // a timed layer is queued behind a host function that holds the stream until all of it
    // is queued, so the events time the kernels and not the host's launch gaps
    int hold_flag = 0;
    auto run_layer = [&](int l, bool timed) {
        auto mark = [&](int k) {
            if (timed) DRV_CUDA(cudaEventRecord(ev[k], 0));
        };
        if (timed) {
            hold_flag = 0;
            DRV_CUDA(cudaLaunchHostFunc(0, LaunchTimer::hold, &hold_flag));
        }
        mark(0);
        DRV_LIB(ternocl_moe_decode_gate_up(dIds, dX, gate[l].dB, gate[l].dS, up[l].dB, up[l].dS, dH, G, I, H, TOPK, E,
                                           dt, nullptr));
        mark(1);
        if (fused) {
            DRV_LIB(ternocl_moe_decode_down_sum(dIds, dH, dRW, down[l].dB, down[l].dS, dO, T, H, I, TOPK, E, dt, nullptr));
            mark(2);
            return;
        }
        DRV_LIB(ternocl_moe_decode_down(dIds, dH, dRW, down[l].dB, down[l].dS, dY, G, H, I, E, dt, nullptr));
        mark(2);
        DRV_LIB(ternocl_moe_decode_reduce(dY, dO, T, H, TOPK, dt, nullptr));
        mark(3);
    };

    // correctness on layer 0
    run_layer(0, false);
    DRV_CUDA(cudaDeviceSynchronize());
    std::vector<uint16_t> O((size_t)T * H);
    DRV_CUDA(cudaMemcpy(O.data(), dO, O.size() * 2, cudaMemcpyDeviceToHost));
    double max_err = 0.0, max_ref = 0.0;
    for (int t = 0; t < T; ++t) {
        std::vector<double> o(H, 0.0);
        for (int j = 0; j < TOPK; ++j) {
            const int g = t * TOPK + j, e = ids[g];
            std::vector<double> h(I);
#pragma omp parallel for
            for (int n = 0; n < I; ++n) {
                double sg = 0.0, su = 0.0;
                for (int k = 0; k < H; ++k) {
                    const double x = tof(X[(size_t)t * H + k]);
                    sg += x * gate[0].w(e, k, n);
                    su += x * up[0].w(e, k, n);
                }
                h[n] = tof(fromf((float)(sg / (1.0 + std::exp(-sg)) * su)));
            }
#pragma omp parallel for
            for (int n = 0; n < H; ++n) {
                double s = 0.0;
                for (int k = 0; k < I; ++k) s += h[k] * down[0].w(e, k, n);
                o[n] += s * tof(RW[g]);
            }
        }
        for (int n = 0; n < H; ++n) {
            max_ref = std::max(max_ref, std::fabs(o[n]));
            max_err = std::max(max_err, std::fabs(o[n] - tof(O[(size_t)t * H + n])));
        }
    }
    const double rel = max_err / std::max(max_ref, 1e-30);
    std::cout << "check: max_abs_err " << std::scientific << std::setprecision(3) << max_err << " (max |ref| " << max_ref
              << ", rel " << rel << ") " << (rel < 1e-2 ? "PASS" : "FAIL") << std::fixed << "\n";
    check_device_error();

    for (int w = 0; w < 50; ++w)
        for (int l = 0; l < sets; ++l) run_layer(l, false);
    DRV_CUDA(cudaDeviceSynchronize());
    const int n_ev = fused ? 2 : 3;
    std::vector<std::vector<double>> tk(3);
    for (int it = 0; it < iters; ++it)
        for (int l = 0; l < sets; ++l) {
            run_layer(l, true);
            __atomic_store_n(&hold_flag, 1, __ATOMIC_RELEASE);
            DRV_CUDA(cudaEventSynchronize(ev[n_ev]));
            for (int k = 0; k < n_ev; ++k) {
                float ms = 0.0f;
                DRV_CUDA(cudaEventElapsedTime(&ms, ev[k], ev[k + 1]));
                tk[k].push_back(ms * 1e3);
            }
        }
    auto med = [](std::vector<double> v) {
        if (v.empty()) return 0.0;
        std::sort(v.begin(), v.end());
        return v[v.size() / 2];
    };
    std::vector<int> uniq(ids.begin(), ids.end());
    std::sort(uniq.begin(), uniq.end());
    const double ne = (double)(std::unique(uniq.begin(), uniq.end()) - uniq.begin());
    const double gu_bytes = ne * 2.0 * ((double)H / 16 * I * 4 + (double)H / kGS * I * 2);
    const double dn_bytes = ne * ((double)I / 16 * H * 4 + (double)I / kGS * H * 2);
    const double a = med(tk[0]), b = med(tk[1]), c = med(tk[2]);
    const double gib = 1024.0 * 1024.0 * 1024.0;
    std::cout << std::setprecision(2) << "gate_up " << a << " us (" << gu_bytes / (a * 1e-6) / gib << " GiB/s)  "
              << (fused ? "down_sum " : "down ") << b << " us (" << dn_bytes / (b * 1e-6) / gib << " GiB/s)  reduce " << c
              << " us  | layer " << a + b + c << " us, " << (gu_bytes + dn_bytes) / ((a + b + c) * 1e-6) / gib
              << " GiB/s, x48 layers = " << 48 * (a + b + c) * 1e-3 << " ms\n";
    check_device_error();
    for (auto &e : ev) cudaEventDestroy(e);
    for (int l = 0; l < sets; ++l)
        for (auto *pp : {&gate, &up, &down}) {
            cudaFree((*pp)[l].dB);
            cudaFree((*pp)[l].dS);
        }
    for (void *p : {(void *)dX, (void *)dRW, (void *)dIds, dH, dO, (void *)dY}) cudaFree(p);
    return 0;
}
