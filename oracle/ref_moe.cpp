// Test infrastructure, not product code (see ref_int2.cpp).  Exports the MoE prefill
// driver's host pieces that the oracle's token reference is built from:
//   Proj::w     int2_moe/prefill.cpp:56-66  weight (e, k, n) of a [E, K/16, N] int2
//               projection with [E, K/128, N] scales (the decode driver's Proj,
//               int2_moe/main.cpp:59-71, is the same function)
//   fill_proj   int2_moe/prefill.cpp:69-79  the driver's expert-weight generator
// The driver's own token check (int2_moe/prefill.cpp:291-310) runs inline in its main(),
// after the OpenCL run, so it cannot be called; the oracle restates it over these pieces.
#define main ternocl_ref_moe_main
#include "int2_moe/prefill.cpp"
#undef main

extern "C" {
// W[e][k][n] = Proj::w(e, k, n) for every element (float, the driver's own arithmetic).
void ref_moe_dequant(const uint32_t *B, const uint16_t *S, int E, int K, int N, float *W) {
    Proj p;
    p.E = E, p.K = K, p.N = N;
    p.B.assign(B, B + p.b_words());
    p.S.resize(p.s_elems());
    std::memcpy(p.S.data(), S, p.s_elems() * sizeof(uint16_t));
    for (int e = 0; e < E; ++e)
        for (int k = 0; k < K; ++k)
            for (int n = 0; n < N; ++n) W[((size_t)e * K + k) * N + n] = p.w(e, k, n);
}

// One projection from a std::mt19937(seed) stream, as the driver fills its first one.
void ref_moe_fill(int E, int K, int N, unsigned seed, uint32_t *B, uint16_t *S) {
    Proj p;
    p.E = E, p.K = K, p.N = N;
    std::mt19937 rng(seed);
    fill_proj(p, rng);
    std::memcpy(B, p.B.data(), p.b_words() * sizeof(uint32_t));
    std::memcpy(S, p.S.data(), p.s_elems() * sizeof(uint16_t));
}
}
