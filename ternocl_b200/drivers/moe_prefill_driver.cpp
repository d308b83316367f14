// Command-line driver of the int2 MoE prefill layer, with the flags and stdout lines of
// int2_moe/prefill.cpp (:81-354): T tokens routed to TOPK of E random ternary experts
// (skewed: expert e drawn with weight 1 / (1 + e/8), without repetition; gate weights
// U(0.05, 1) normalised per token), one layer = route, gather, up, gate (SiLU(gate) * up),
// down (fp32 out), combine, a double-precision host reference on the first --check
// tokens ("check (...): ... PASS|FAIL") and per-kernel device times over --sets
// distinct weight copies (median per kernel, "| layer X us, T TFLOPS, x48 = Y ms").
// --int8 Q runs the int8-activation layer of int2_moe_prefill_int8.cl (prefill.cpp:232-265,
// check bound 5e-2): Q = 0 quantises the T token rows and gathers the int8 rows with their
// scales (gather_q); Q = 1 gathers the fp16 rows and quantises the G routed rows (the
// reference quantises those inside its GEMM; the codes are the same, a * SA being exact in
// fp32).  H is quantised before down in both.
#include <fstream>

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

// one expert by weight, then its weight is removed (sampling without repetition)
int draw(std::vector<double> &w) {
    double tot = 0.0;
    for (double x : w) tot += x;
    double u = (double)rnd_uniform(0.0f, 1.0f) * tot;
    int last = -1;
    for (int e = 0; e < (int)w.size(); ++e) {
        if (w[e] <= 0.0) continue;
        last = e;
        if (u < w[e]) break;
        u -= w[e];
    }
    w[last] = 0.0;
    return last;
}

}  // namespace

int main(int argc, char **argv) {
    int T = 1024, E = 128, TOPK = 8, H = 2048, I = 768, sets = 8, iters = 10, check = 4, qmode = -1;
    std::string dump_up;
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
        else if (f.is("--check") && v) check = f.ival();
        else if (f.is("--dump-up") && v) dump_up = f.value();
        else if (f.is("--seed") && v) seed_base() = (uint64_t)std::strtoull(f.value(), nullptr, 10), seed_fixed() = true;
        else if (f.is("--dtype") && v) {
            if (!parse_dtype(f)) {
                std::cerr << "--dtype fp16|bf16\n";
                return 1;
            }
        } else if ((f.is("--tile") || f.is("--dir")) && v) f.ignore(true);
        else if (f.is("--int8") && v) {
            qmode = f.ival();
            if (qmode != 0 && qmode != 1) {
                std::cerr << "--int8 0|1\n";
                return 1;
            }
        } else {
            std::cerr << "usage: " << argv[0]
                      << " [--t T] [--e E] [--topk K] [--h H] [--i I] [--sets S] [--iters N] [--check C]"
                         " [--int8 qmode] [--dtype fp16|bf16] [--seed S] [--dump-up file]"
                         "  (accepted and ignored: --tile --dir)\n";
            return 1;
        }
    }
    if (T < 1 || E < 1 || TOPK < 1 || TOPK > E || H % kGS || I % kGS || H % 16 || I % 16 || sets < 1 || iters < 1) {
        std::cerr << "need 1 <= topk <= E, H and I multiples of 128\n";
        return 1;
    }
    seed_base() = seed_fixed() ? seed_base() : 42;  // the reference seeds its layer with 42
    seed_fixed() = true;
    const int G = T * TOPK;
    const int dt = dt_code();
    const bool int8 = qmode >= 0;
    std::cout << "Prefill: T=" << T << " E=" << E << " topk=" << TOPK << " H=" << H << " I=" << I << " tile "
              << ternocl_moe_rows_per_tile() << (int8 ? "x128 (tcgen05 grouped s8 x s2 GEMM, sm_100a)"
                                                      : "x256 (tcgen05 grouped GEMM, sm_100a)")
              << " dtype=" << dt_name() << (int8 ? " int8 activations, qmode " + std::to_string(qmode) : "") << "\n";
    report_ignored(f);

    Proj gate{E, H, I, {}, {}}, up{E, H, I, {}, {}}, down{E, I, H, {}, {}};
    fill_proj(gate);
    fill_proj(up);
    fill_proj(down);
    // --sets copies of the same layer's weights at distinct addresses
    std::vector<Proj> lg(sets, gate), lu(sets, up), ld(sets, down);
    for (int l = 0; l < sets; ++l)
        for (Proj *p : {&lg[l], &lu[l], &ld[l]}) {
            p->dB = to_device(p->B);
            p->dS = to_device(p->S);
            p->B.clear();
            p->S.clear();
        }

    std::vector<uint16_t> X((size_t)T * H), RW(G);
    std::vector<int32_t> ids(G);
    for (auto &x : X) x = fromf(rnd_uniform(-1.0f, 1.0f));
    std::vector<double> pw(E);
    for (int e = 0; e < E; ++e) pw[e] = 1.0 / (1.0 + e / 8.0);
    for (int t = 0; t < T; ++t) {
        std::vector<double> w = pw;
        std::vector<float> r(TOPK);
        float sum = 0.0f;
        for (int j = 0; j < TOPK; ++j) {
            ids[(size_t)t * TOPK + j] = draw(w);
            sum += (r[j] = rnd_uniform(0.05f, 1.0f));
        }
        for (int j = 0; j < TOPK; ++j) RW[(size_t)t * TOPK + j] = fromf(r[j] / sum);
    }
    uint16_t *dX = to_device(X), *dRW = to_device(RW);
    int32_t *dIds = to_device(ids);
    int32_t *dMeta = (int32_t *)device_alloc((size_t)(2 * E + 2) * 4);
    int32_t *dPerm = (int32_t *)device_alloc((size_t)G * 4), *dInv = (int32_t *)device_alloc((size_t)G * 4);
    void *dXs = device_alloc((size_t)G * H * 2), *dU = device_alloc((size_t)G * I * 2);
    void *dH = device_alloc((size_t)G * I * 2), *dO = device_alloc((size_t)T * H * 2);
    float *dY = (float *)device_alloc((size_t)G * H * 4);
    const int rpt = ternocl_moe_rows_per_tile();
    // int8 path: codes and per-(128-group, row) scales, rows padded to LDSA = 32
    int8_t *dXq = nullptr, *dXsq = nullptr, *dHq = nullptr;
    void *dSAt = nullptr, *dSA1 = nullptr, *dSA2 = nullptr;
    if (int8) {
        dXq = (int8_t *)device_alloc((size_t)T * H);
        dXsq = (int8_t *)device_alloc((size_t)G * H);
        dHq = (int8_t *)device_alloc((size_t)G * I);
        dSAt = device_alloc((size_t)H / kGS * ternocl_int8_ldsa(T) * 2);
        dSA1 = device_alloc((size_t)H / kGS * ternocl_int8_ldsa(G) * 2);
        dSA2 = device_alloc((size_t)I / kGS * ternocl_int8_ldsa(G) * 2);
    }
    std::vector<const char *> names = {"route", "gather", "up", "gate", "down", "combine"};
    if (int8 && qmode == 0) names = {"route", "quant_x", "gather_q", "up", "gate", "quant_h", "down", "combine"};
    if (int8 && qmode == 1) names = {"route", "gather", "quant_x", "up", "gate", "quant_h", "down", "combine"};
    const int n_k = (int)names.size();

    cudaEvent_t ev[9];
    for (auto &e : ev) DRV_CUDA(cudaEventCreate(&e));
    // a timed layer is queued behind a host function that holds the stream until all of it
    // is queued, so the events time the kernels and not the host's launch gaps
    int hold_flag = 0;
    auto run_layer = [&](int l, bool timed) {
        int k = 0;
        auto mark = [&]() {
            if (timed) DRV_CUDA(cudaEventRecord(ev[k], 0));
            ++k;
        };
        if (timed) {
            hold_flag = 0;
            DRV_CUDA(cudaLaunchHostFunc(0, LaunchTimer::hold, &hold_flag));
        }
        mark();
        DRV_LIB(ternocl_moe_route(dIds, dMeta, dPerm, dInv, G, E, rpt, nullptr));
        mark();
        if (int8) {
            if (qmode == 0) {
                DRV_LIB(ternocl_int8_quant_a(dX, dSAt, dXq, T, H, dt, nullptr));
                mark();
                DRV_LIB(ternocl_moe_gather_q(dXq, dSAt, dPerm, dXsq, dSA1, T, G, H, TOPK, nullptr));
            } else {
                DRV_LIB(ternocl_moe_gather(dX, dPerm, dXs, G, H, TOPK, nullptr));
                mark();
                DRV_LIB(ternocl_int8_quant_a(dXs, dSA1, dXsq, G, H, dt, nullptr));
            }
            mark();
            DRV_LIB(ternocl_moe_gemm_i8(dMeta, nullptr, dXsq, dSA1, lu[l].dB, lu[l].dS, dU, nullptr, G, I, H, E, dt, 0,
                                        0, 0, nullptr));
            mark();
            DRV_LIB(ternocl_moe_gemm_i8(dMeta, nullptr, dXsq, dSA1, lg[l].dB, lg[l].dS, dH, dU, G, I, H, E, dt, 1, 0,
                                        0, nullptr));
            mark();
            DRV_LIB(ternocl_int8_quant_a(dH, dSA2, dHq, G, I, dt, nullptr));
            mark();
            DRV_LIB(ternocl_moe_gemm_i8(dMeta, nullptr, dHq, dSA2, ld[l].dB, ld[l].dS, dY, nullptr, G, H, I, E, dt, 0,
                                        1, 0, nullptr));
        } else {
            DRV_LIB(ternocl_moe_gather(dX, dPerm, dXs, G, H, TOPK, nullptr));
            mark();
            DRV_LIB(ternocl_moe_gemm(dMeta, dXs, lu[l].dB, lu[l].dS, dU, nullptr, G, I, H, E, dt, 0, 0, nullptr));
            mark();
            DRV_LIB(ternocl_moe_gemm(dMeta, dXs, lg[l].dB, lg[l].dS, dH, dU, G, I, H, E, dt, 1, 0, nullptr));
            mark();
            DRV_LIB(ternocl_moe_gemm(dMeta, dH, ld[l].dB, ld[l].dS, dY, nullptr, G, H, I, E, dt, 0, 1, nullptr));
        }
        mark();
        DRV_LIB(ternocl_moe_combine(dY, dInv, dRW, dO, T, H, TOPK, dt, nullptr));
        mark();
    };

    run_layer(0, false);
    DRV_CUDA(cudaDeviceSynchronize());
    if (!dump_up.empty()) {
        std::vector<uint16_t> u((size_t)G * I);
        DRV_CUDA(cudaMemcpy(u.data(), dU, u.size() * 2, cudaMemcpyDeviceToHost));
        std::ofstream(dump_up, std::ios::binary).write((const char *)u.data(), (std::streamsize)(u.size() * 2));
    }
    std::vector<uint16_t> O((size_t)T * H);
    DRV_CUDA(cudaMemcpy(O.data(), dO, O.size() * 2, cudaMemcpyDeviceToHost));
    // host reference of the first tokens (double sums; the device's DT roundings of up and H)
    const int nchk = std::min(T, check);
    double max_err = 0.0, max_ref = 0.0;
#pragma omp parallel for reduction(max : max_err, max_ref)
    for (int t = 0; t < nchk; ++t) {
        std::vector<double> o(H, 0.0);
        std::vector<double> h(I);
        for (int j = 0; j < TOPK; ++j) {
            const int g = t * TOPK + j, e = ids[g];
            for (int n = 0; n < I; ++n) {
                double sg = 0.0, su = 0.0;
                for (int k = 0; k < H; ++k) {
                    const double x = tof(X[(size_t)t * H + k]);
                    sg += x * gate.w(e, k, n);
                    su += x * up.w(e, k, n);
                }
                const double silu = sg / (1.0 + std::exp(-sg));
                h[n] = tof(fromf((float)(silu * tof(fromf((float)su)))));
            }
            for (int n = 0; n < H; ++n) {
                double s = 0.0;
                for (int k = 0; k < I; ++k) s += h[k] * down.w(e, k, n);
                o[n] += s * tof(RW[g]);
            }
        }
        for (int n = 0; n < H; ++n) {
            max_ref = std::max(max_ref, std::fabs(o[n]));
            max_err = std::max(max_err, std::fabs(o[n] - tof(O[(size_t)t * H + n])));
        }
    }
    const double rel = max_err / std::max(max_ref, 1e-30);
    std::cout << "check (" << nchk << " tokens): max_abs_err " << std::scientific << std::setprecision(3) << max_err
              << " (max |ref| " << max_ref << ", rel " << rel << ") " << (rel < (int8 ? 5e-2 : 1e-2) ? "PASS" : "FAIL")
              << std::fixed
              << "\n";
    check_device_error();

    for (int w = 0; w < 10; ++w)
        for (int l = 0; l < sets; ++l) run_layer(l, false);
    DRV_CUDA(cudaDeviceSynchronize());
    std::vector<std::vector<double>> tk(n_k);
    for (int it = 0; it < iters; ++it)
        for (int l = 0; l < sets; ++l) {
            run_layer(l, true);
            __atomic_store_n(&hold_flag, 1, __ATOMIC_RELEASE);
            DRV_CUDA(cudaEventSynchronize(ev[n_k]));
            for (int k = 0; k < n_k; ++k) {
                float ms = 0.0f;
                DRV_CUDA(cudaEventElapsedTime(&ms, ev[k], ev[k + 1]));
                tk[k].push_back(ms * 1e3);
            }
        }
    double total = 0.0;
    std::cout << std::setprecision(1);
    for (int k = 0; k < n_k; ++k) {
        std::sort(tk[k].begin(), tk[k].end());
        const double m = tk[k][tk[k].size() / 2];
        total += m;
        std::cout << names[k] << " " << m << " us  ";
    }
    const double flops = 2.0 * G * (2.0 * H * I + (double)I * H);
    std::cout << "| layer " << total << " us, " << flops / (total * 1e-6) / 1e12 << " TFLOPS, x48 = " << 48 * total / 1e3
              << " ms\n";
    check_device_error();
    for (auto &e : ev) cudaEventDestroy(e);
    for (int l = 0; l < sets; ++l)
        for (Proj *p : {&lg[l], &lu[l], &ld[l]}) {
            cudaFree(p->dB);
            cudaFree(p->dS);
        }
    for (void *p : {(void *)dX, (void *)dRW, (void *)dIds, (void *)dMeta, (void *)dPerm, (void *)dInv, dXs, dU, dH,
                    dO, (void *)dY, (void *)dXq, (void *)dXsq, (void *)dHq, dSAt, dSA1, dSA2})
        cudaFree(p);
    return 0;
}
