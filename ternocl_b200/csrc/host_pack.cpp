// Host-side weight packers of libternocl (no device work): BITCOS and the int1
// select layout.  They produce the reference layouts bit for bit:
//   BITCOS  common/bitcos.hpp:1-8 (layout), :31-78 (random packer), :81-94 (slice ranks)
//   int1    int1_fp16_upcvt/main.cpp:76-92 (per-column order -> sel layout)
#include <omp.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#include "ternocl.h"

namespace {

constexpr size_t kPadWords = 4;  // the GEMVs' sign window reads up to two words past a run

// Assemble bitmap | offsets | signs | pad from a bitmap and a per-column sign-bit
// source.  signs_of(n, words_out) fills column n's sign words.
template <class SignFill>
size_t assemble(const std::vector<uint32_t> &bmp, int K, int N, uint32_t *out, size_t cap,
                SignFill &&signs_of) {
    const size_t bw = (size_t)(K / 32) * N;
    std::vector<uint32_t> nnz(N, 0), off(N, 0);
#pragma omp parallel for
    for (int n = 0; n < N; ++n) {
        uint32_t s = 0;
        for (int kp = 0; kp < K / 32; ++kp) s += (uint32_t)__builtin_popcount(bmp[(size_t)kp * N + n]);
        nnz[n] = s;
    }
    size_t words = 0;
    for (int n = 0; n < N; ++n) {
        off[n] = (uint32_t)words;
        words += (nnz[n] + 31) / 32;
    }
    const size_t total = bw + N + words + kPadWords;
    if (!out || cap < total) return total;
    std::copy(bmp.begin(), bmp.end(), out);
    std::copy(off.begin(), off.end(), out + bw);
    std::memset(out + bw + N, 0, (words + kPadWords) * sizeof(uint32_t));
    signs_of(out + bw + N, nnz, off);
    return total;
}

}  // namespace

extern "C" {

// Same generator streams as the reference packer: bitmap bits from one mt19937 per
// OpenMP thread seeded seed*7919 + thread (static schedule over bitmap words), sign
// words from mt19937(seed*104729 + 17 + thread) over columns, tail bits cleared.
size_t ternocl_bitcos_random(int K, int N, double z, uint64_t seed, uint32_t *out, size_t cap) {
    if (K <= 0 || N <= 0 || K % 32) return 0;
    const size_t bw = (size_t)(K / 32) * N;
    std::vector<uint32_t> bmp(bw);
    const double t = (1.0 - z) * 4294967296.0;
    const uint32_t thr = (uint32_t)(t > 4294967295.0 ? 4294967295.0 : t);
#pragma omp parallel
    {
        std::mt19937 g((uint32_t)(seed * 7919u + (uint64_t)omp_get_thread_num()));
#pragma omp for schedule(static)
        for (long long i = 0; i < (long long)bw; ++i) {
            uint32_t w = 0;
            for (int c = 0; c < 32; ++c) w |= (uint32_t)(g() < thr) << c;
            bmp[i] = w;
        }
    }
    return assemble(bmp, K, N, out, cap,
                    [&](uint32_t *sg, const std::vector<uint32_t> &nnz, const std::vector<uint32_t> &off) {
#pragma omp parallel
                        {
                            std::mt19937 g((uint32_t)(seed * 104729u + 17u + (uint64_t)omp_get_thread_num()));
#pragma omp for schedule(static)
                            for (int n = 0; n < N; ++n) {
                                const uint32_t nw = (nnz[n] + 31) / 32;
                                for (uint32_t w = 0; w < nw; ++w) {
                                    uint32_t v = g();
                                    const uint32_t bits = std::min<uint32_t>(32, nnz[n] - 32 * w);
                                    if (bits < 32) v &= (1u << bits) - 1u;
                                    sg[off[n] + w] = v;
                                }
                            }
                        }
                    });
}

// codes [K, N] row-major in {-1, 0, +1} -> BITCOS buffer.
size_t ternocl_bitcos_pack(const int8_t *codes, int K, int N, uint32_t *out, size_t cap) {
    if (!codes || K <= 0 || N <= 0 || K % 32) return 0;
    const size_t bw = (size_t)(K / 32) * N;
    std::vector<uint32_t> bmp(bw);
#pragma omp parallel for
    for (long long i = 0; i < (long long)bw; ++i) {
        const int kp = (int)(i / N), n = (int)(i % N);
        uint32_t w = 0;
        for (int c = 0; c < 32; ++c) w |= (uint32_t)(codes[(size_t)(32 * kp + c) * N + n] != 0) << c;
        bmp[i] = w;
    }
    return assemble(bmp, K, N, out, cap,
                    [&](uint32_t *sg, const std::vector<uint32_t> &, const std::vector<uint32_t> &off) {
#pragma omp parallel for
                        for (int n = 0; n < N; ++n) {
                            uint32_t rank = 0;
                            for (int k = 0; k < K; ++k) {
                                const int8_t c = codes[(size_t)k * N + n];
                                if (!c) continue;
                                if (c < 0) sg[off[n] + rank / 32] |= 1u << (rank % 32);
                                ++rank;
                            }
                        }
                    });
}

int ternocl_bitcos_slice_ranks(const uint32_t *buf, int K, int N, int ls, uint32_t *out) {
    if (!buf || K <= 0 || N <= 0 || K % 32 || ls < 1) return TERNOCL_ERR_ARG;
    if (ls == 1) return TERNOCL_OK;
    if (!out) return TERNOCL_ERR_ARG;
    const int slice_k = (K + ls - 1) / ls;
#pragma omp parallel for
    for (int n = 0; n < N; ++n) {
        uint32_t s = 0;
        int kp = 0;
        for (int sl = 1; sl < ls; ++sl) {
            for (; kp < sl * slice_k / 32; ++kp) s += (uint32_t)__builtin_popcount(buf[(size_t)kp * N + n]);
            out[(size_t)(sl - 1) * N + n] = s;
        }
    }
    return TERNOCL_OK;
}

int ternocl_int1_to_sel(const uint32_t *B, uint32_t *out, int K, int N) {
    if (!B || !out) return TERNOCL_ERR_ARG;
    if (K <= 0 || N <= 0 || K % 32 || N % 16) return TERNOCL_ERR_SHAPE;
#pragma omp parallel for collapse(2)
    for (int kp = 0; kp < K / 32; ++kp)
        for (int n0 = 0; n0 < N; n0 += 16) {
            const uint32_t *src = B + (size_t)kp * N + n0;
            for (int p = 0; p < 16; ++p) {
                uint32_t w = 0;
                for (int j = 0; j < 32; ++j) w |= ((src[j >> 1] >> ((j & 1) * 16 + p)) & 1u) << j;
                out[(size_t)kp * N + n0 + p] = w;
            }
        }
    return TERNOCL_OK;
}

}  // extern "C"
