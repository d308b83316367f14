/* Test oracle: plain-C restatement of the reference host gold (see oracle.h).
 * TEST INFRASTRUCTURE ONLY -- never linked into the product.
 *
 * Each function restates the cited reference code with the same floating-point
 * operation sequence (built with -ffp-contract=off, like oracle/_ref), so that the
 * two agree bit for bit on identical inputs; tests/test_oracle_pins.py checks that. */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define GS 128

/* common/dt16.hpp:18-28 */
float orc_tof(uint16_t h, int bf16) {
    if (bf16) {
        const uint32_t u = (uint32_t)h << 16;
        float f;
        memcpy(&f, &u, 4);
        return f;
    }
    _Float16 x;
    memcpy(&x, &h, 2);
    return (float)x;
}

/* common/dt16.hpp:30-42: bf16 round-to-nearest-even with NaN quieting; fp16 IEEE RNE */
uint16_t orc_fromf(float f, int bf16) {
    if (bf16) {
        uint32_t u;
        memcpy(&u, &f, 4);
        if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
        u += 0x7fffu + ((u >> 16) & 1u);
        return (uint16_t)(u >> 16);
    }
    const _Float16 x = (_Float16)f;
    uint16_t h;
    memcpy(&h, &x, 2);
    return h;
}

/* int2_fp16_upcvt/main.cpp:76: 2-bit two's complement code */
static int code_to_value(uint32_t c) { return (int)(int8_t)((int8_t)(c << 6) >> 6); }

int orc_int2_value(const uint32_t *B, int N, int k, int n) {
    return code_to_value((B[(size_t)(k / 16) * N + n] >> (2 * (k % 16))) & 3u);
}

/* int2_fp16_upcvt/main.cpp:79-98 */
void orc_int2_gold(const uint16_t *A, const uint32_t *B, const uint16_t *S, float *C, int M, int K,
                   int N, int bf16) {
    const int groups = K / GS;
#pragma omp parallel for collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int g = 0; g < groups; ++g) {
                float partial = 0.0f;
                for (int p = 0; p < GS; ++p) {
                    const int ik = g * GS + p;
                    const uint32_t code = (B[(size_t)(ik / 16) * N + j] >> (2 * (ik % 16))) & 3u;
                    const int bv = code_to_value(code);
                    if (bv) partial += orc_tof(A[(size_t)i * K + ik], bf16) * (float)bv;
                }
                acc += partial * orc_tof(S[(size_t)g * N + j], bf16);
            }
            C[(size_t)i * N + j] = acc;
        }
}

/* int1_fp16_upcvt/main.cpp:76: VNNI2 bit order, even rows in the low half */
int orc_int1_bit_pos(int k) {
    const int r = k % 32;
    return (r & 1) * 16 + r / 2;
}

/* int1_fp16_upcvt/main.cpp:95-114 (bit 1 = -1) */
void orc_int1_gold(const uint16_t *A, const uint32_t *B, const uint16_t *S, float *C, int M, int K,
                   int N, int bf16) {
    const int groups = K / GS;
#pragma omp parallel for collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int g = 0; g < groups; ++g) {
                float partial = 0.0f;
                for (int p = 0; p < GS; ++p) {
                    const int ik = g * GS + p;
                    const int neg = (B[(size_t)(ik / 32) * N + j] >> orc_int1_bit_pos(ik)) & 1u;
                    const float a = orc_tof(A[(size_t)i * K + ik], bf16);
                    partial += neg ? -a : a;
                }
                acc += partial * orc_tof(S[(size_t)g * N + j], bf16);
            }
            C[(size_t)i * N + j] = acc;
        }
}

/* int1_fp16_upcvt/main.cpp:80-92: word (kp, n0+p) bit j = (row 32kp+2p+(j&1), col n0+j/2) */
void orc_int1_to_sel(const uint32_t *B, uint32_t *O, int K, int N) {
#pragma omp parallel for collapse(2)
    for (int kp = 0; kp < K / 32; ++kp)
        for (int n0 = 0; n0 < N; n0 += 16) {
            const uint32_t *src = B + (size_t)kp * N + n0;
            for (int p = 0; p < 16; ++p) {
                uint32_t w = 0;
                for (int j = 0; j < 32; ++j) w |= ((src[j >> 1] >> ((j & 1) * 16 + p)) & 1u) << j;
                O[(size_t)kp * N + n0 + p] = w;
            }
        }
}

/* int2_via_int2_x_int8_dpas/main.cpp:79: SA row pitch */
int orc_int8_ldsa(int M) { return (M + 31) & ~31; }

/* int2_via_int2_x_int8_dpas/main.cpp:82-91: SA = DT(127 / max(FLT_EPSILON, absmax)) */
void orc_int8_scale_a(const uint16_t *A, uint16_t *SA, int M, int K, int bf16) {
    const int ld = orc_int8_ldsa(M);
#pragma omp parallel for
    for (int m = 0; m < M; ++m)
        for (int g = 0; g < K / GS; ++g) {
            float mx = FLT_EPSILON;
            for (int p = 0; p < GS; ++p) {
                const float v = fabsf(orc_tof(A[(size_t)m * K + g * GS + p], bf16));
                mx = (mx < v) ? v : mx; /* std::max(mx, v) */
            }
            SA[(size_t)g * ld + m] = orc_fromf(127.0f / mx, bf16);
        }
}

/* int2_via_int2_x_int8_dpas/main.cpp:97-103: q = sat_int8(lrintf(A * SA)), RTE */
void orc_int8_quant(const uint16_t *A, const uint16_t *SA, int8_t *Q, int M, int K, int bf16) {
    const int ld = orc_int8_ldsa(M);
#pragma omp parallel for
    for (int m = 0; m < M; ++m)
        for (int k = 0; k < K; ++k) {
            long v = lrintf(orc_tof(A[(size_t)m * K + k], bf16) *
                            orc_tof(SA[(size_t)(k / GS) * ld + m], bf16));
            v = v < -128L ? -128L : (v > 127L ? 127L : v);
            Q[(size_t)m * K + k] = (int8_t)v;
        }
}

/* int2_via_int2_x_int8_dpas/main.cpp:109-114: int32 dot per (m, group, n); D[(m*G + g)*N + n] */
void orc_int8_group_dots(const int8_t *Q, const uint32_t *B, int32_t *D, int M, int K, int N) {
    const int groups = K / GS;
#pragma omp parallel for collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j)
            for (int g = 0; g < groups; ++g) {
                int32_t dot = 0;
                for (int p = 0; p < GS; ++p) {
                    const int ik = g * GS + p;
                    const uint32_t code = (B[(size_t)(ik / 16) * N + j] >> (2 * (ik % 16))) & 3u;
                    dot += (int)Q[(size_t)i * K + ik] * code_to_value(code);
                }
                D[((size_t)i * groups + g) * N + j] = dot;
            }
}

/* int2_via_int2_x_int8_dpas/main.cpp:94-121 */
void orc_int8_gold(const uint16_t *A, const uint32_t *B, const uint16_t *SA, const uint16_t *SB,
                   float *C, int M, int K, int N, int bf16) {
    const int groups = K / GS, ld = orc_int8_ldsa(M);
    int8_t *q = (int8_t *)malloc((size_t)M * K);
    orc_int8_quant(A, SA, q, M, K, bf16);
#pragma omp parallel for collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int g = 0; g < groups; ++g) {
                int32_t dot = 0;
                for (int p = 0; p < GS; ++p) {
                    const int ik = g * GS + p;
                    const uint32_t code = (B[(size_t)(ik / 16) * N + j] >> (2 * (ik % 16))) & 3u;
                    dot += (int)q[(size_t)i * K + ik] * code_to_value(code);
                }
                const float sa = orc_tof(SA[(size_t)g * ld + i], bf16);
                const float inv = sa == 0.0f ? 0.0f : 1.0f / sa;
                acc += (float)dot * (orc_tof(SB[(size_t)g * N + j], bf16) * inv);
            }
            C[(size_t)i * N + j] = acc;
        }
    free(q);
}

/* int2_via_int2_x_int8_dpas/main.cpp:261-272 (the fill's fake quantisation, then SA again) */
void orc_int8_fake_quant(uint16_t *A, uint16_t *SA, int M, int K, float offgrid, int bf16) {
    const int ld = orc_int8_ldsa(M);
    orc_int8_scale_a(A, SA, M, K, bf16);
#pragma omp parallel for
    for (int m = 0; m < M; ++m)
        for (int k = 0; k < K; ++k) {
            const float sa = orc_tof(SA[(size_t)(k / GS) * ld + m], bf16);
            long v = lrintf(orc_tof(A[(size_t)m * K + k], bf16) * sa);
            v = v < -128L ? -128L : (v > 127L ? 127L : v);
            const float off = v >= 0 ? offgrid : -offgrid;
            A[(size_t)m * K + k] = orc_fromf(((float)v + off) * (1.0f / sa), bf16);
        }
    orc_int8_scale_a(A, SA, M, K, bf16);
}

/* common/bitcos.hpp:17-25: bitmap [K/32][N] | offsets [N] | signs | pad */
size_t orc_bitcos_words(const uint32_t *buf, int K, int N) {
    /* total words = bitmap + offsets + sign words + 4 pad words (bitcos.hpp:27,59) */
    const size_t bw = (size_t)(K / 32) * N;
    size_t words = 0;
    for (int n = 0; n < N; ++n) {
        uint32_t s = 0;
        for (int kp = 0; kp < K / 32; ++kp) s += (uint32_t)__builtin_popcount(buf[(size_t)kp * N + n]);
        words += (s + 31) / 32;
    }
    return bw + N + words + 4;
}

/* common/bitcos.hpp:97-106, all columns */
void orc_bitcos_decode(const uint32_t *buf, int K, int N, int8_t *codes) {
    const size_t bw = (size_t)(K / 32) * N;
#pragma omp parallel for
    for (int n = 0; n < N; ++n) {
        const uint32_t *sg = buf + bw + N + buf[bw + n];
        uint32_t rank = 0;
        for (int k = 0; k < K; ++k) {
            const int p = (buf[(size_t)(k / 32) * N + n] >> (k % 32)) & 1u;
            if (!p) { codes[(size_t)n * K + k] = 0; continue; }
            codes[(size_t)n * K + k] = ((sg[rank / 32] >> (rank % 32)) & 1u) ? -1 : 1;
            ++rank;
        }
    }
}

/* bitcos_fp16_upcvt/main.cpp:64-86 */
void orc_bitcos_gold(const uint16_t *A, const uint32_t *buf, const uint16_t *S, float *C, int M,
                     int K, int N, int bf16) {
    int8_t *codes = (int8_t *)malloc((size_t)K * N);
    orc_bitcos_decode(buf, K, N, codes);
#pragma omp parallel for
    for (int j = 0; j < N; ++j) {
        const int8_t *cj = codes + (size_t)j * K;
        for (int i = 0; i < M; ++i) {
            float acc = 0.0f;
            for (int g = 0; g < K / GS; ++g) {
                float partial = 0.0f;
                for (int p = 0; p < GS; ++p) {
                    const int k = g * GS + p;
                    if (cj[k]) partial += orc_tof(A[(size_t)i * K + k], bf16) * (float)cj[k];
                }
                acc += partial * orc_tof(S[(size_t)g * N + j], bf16);
            }
            C[(size_t)i * N + j] = acc;
        }
    }
    free(codes);
}

/* common/bitcos.hpp:81-94: non-zeros of column n above each slice boundary */
void orc_bitcos_slice_ranks(const uint32_t *buf, int K, int N, int ls, uint32_t *out) {
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
}

/* common/epilogue.hpp:34 (xetla_sigmoid) */
static float sigmoid_ref(float x) { return x <= -10.0f ? 0.0f : 1.0f / (expf(-x) + 1.0f); }

/* common/epilogue.hpp:50-67 */
void orc_epilogue(int postop, int out_f32, const float *acc, const uint16_t *other,
                  const void *bias, void *out, int M, int N, int bf16) {
    const unsigned char *bb = (const unsigned char *)bias;
    unsigned char *ob = (unsigned char *)out;
#pragma omp parallel for
    for (long long i = 0; i < (long long)M * N; ++i) {
        float v = acc[i];
        const int n = (int)(i % N);
        if (postop == 1) v = v * sigmoid_ref(v) * orc_tof(other[i], bf16);
        else if (postop == 2) v += orc_tof(other[i], bf16);
        else if (postop == 3) {
            float b;
            if (out_f32) memcpy(&b, bb + 4 * (size_t)n, 4);
            else { uint16_t h; memcpy(&h, bb + 2 * (size_t)n, 2); b = orc_tof(h, bf16); }
            v += b;
        } else if (postop == 4) v = sigmoid_ref(v);
        if (out_f32) memcpy(ob + 4 * (size_t)i, &v, 4);
        else { const uint16_t h = orc_fromf(v, bf16); memcpy(ob + 2 * (size_t)i, &h, 2); }
    }
}

/* hadamard/hadamard_fwht.cl:62-115.  Per HB block: v = x * sign in fp32, then the
 * log2(HB) radix-2 stages in increasing stride order (the .cl's radix-8 passes do
 * strides 8^p, 2*8^p, 4*8^p, then its trailing radix-2/4 pass the top strides),
 * each stage (a + b, a - b) in fp32, then DT(v * SCALE).  The result of a stage
 * sequence does not depend on how the independent butterflies of a stage are
 * grouped, so this plain loop reproduces the kernel bit for bit. */
int orc_hadamard(const uint16_t *x, const int8_t *signs, uint16_t *y, int rows, int K, int HB,
                 int use_signs, int bf16) {
    if (HB < 256 || HB > 4096 || (HB & (HB - 1)) || K % HB) return -1;
    /* hadamard_fwht.cl:17-31: SCALE = 1/sqrt(HB) as a float literal */
    const float scale = (float)(1.0 / sqrt((double)HB));
    const int bpr = K / HB;
#pragma omp parallel for
    for (long long blk = 0; blk < (long long)rows * bpr; ++blk) {
        float v[4096];
        const size_t off = (size_t)(blk / bpr) * K + (size_t)(blk % bpr) * HB;
        const int8_t *sb = signs + (size_t)(blk % bpr) * HB;
        for (int i = 0; i < HB; ++i) {
            const float a = orc_tof(x[off + i], bf16);
            v[i] = use_signs ? a * (float)sb[i] : a;
        }
        for (int h = 1; h < HB; h <<= 1)
            for (int i = 0; i < HB; ++i)
                if ((i & h) == 0) {
                    const float a = v[i], b = v[i + h];
                    v[i] = a + b;
                    v[i + h] = a - b;
                }
        for (int i = 0; i < HB; ++i) y[off + i] = orc_fromf(v[i] * scale, bf16);
    }
    return 0;
}

/* int2_moe/int2_moe_prefill.cl:29-61 (meta layout [E+1 row offsets | E+1 tile
 * offsets]); the permutation inside an expert is ascending in g here, where the
 * reference's order follows its local atomics. */
void orc_moe_route(const int *ids, int G, int E, int rows_per_tile, int *meta, int *perm, int *inv) {
    int *cnt = (int *)calloc((size_t)E, sizeof(int));
    for (int g = 0; g < G; ++g) cnt[ids[g]]++;
    int r = 0, t = 0;
    for (int e = 0; e < E; ++e) {
        meta[e] = r;
        meta[E + 1 + e] = t;
        r += cnt[e];
        t += (cnt[e] + rows_per_tile - 1) / rows_per_tile;
        cnt[e] = 0;
    }
    meta[E] = r;
    meta[2 * E + 1] = t;
    for (int g = 0; g < G; ++g) {
        const int e = ids[g];
        const int p = meta[e] + cnt[e]++;
        perm[p] = g;
        inv[g] = p;
    }
    free(cnt);
}

/* int2_moe/prefill.cpp:56-66: weight (e, k, n) of a [E, K/16, N] int2 projection */
static float proj_w(const uint32_t *B, const uint16_t *S, int K, int N, int e, int k, int n, int bf16) {
    const uint32_t word = B[((size_t)e * (K / 16) + k / 16) * N + n];
    return (float)code_to_value((word >> (2 * (k % 16))) & 3u) *
           orc_tof(S[((size_t)e * (K / GS) + k / GS) * N + n], bf16);
}

/* W[e][k][n] = proj_w(e, k, n) over a whole [E, K/16, N] projection (the pin of proj_w) */
void orc_moe_dequant(const uint32_t *B, const uint16_t *S, int E, int K, int N, float *W, int bf16) {
    for (int e = 0; e < E; ++e)
        for (int k = 0; k < K; ++k)
            for (int n = 0; n < N; ++n) W[((size_t)e * K + k) * N + n] = proj_w(B, S, K, N, e, k, n, bf16);
}

/* int2_moe/prefill.cpp:291-310: o[n] = sum_j RW[g] * down(h),
 * h = DT(silu(gate.x) * DT(up.x)) in double precision */
void orc_moe_token_ref(const uint16_t *X, const int *ids, const uint16_t *RW, const uint32_t *Bg,
                       const uint16_t *Sg, const uint32_t *Bu, const uint16_t *Su,
                       const uint32_t *Bd, const uint16_t *Sd, int t, int topk, int H, int I,
                       double *o, int bf16) {
    for (int n = 0; n < H; ++n) o[n] = 0.0;
    float *h = (float *)malloc((size_t)I * sizeof(float));
    for (int j = 0; j < topk; ++j) {
        const int g = t * topk + j, e = ids[g];
#pragma omp parallel for
        for (int n = 0; n < I; ++n) {
            double sg = 0.0, su = 0.0;
            for (int k = 0; k < H; ++k) {
                const double x = orc_tof(X[(size_t)t * H + k], bf16);
                sg += x * proj_w(Bg, Sg, H, I, e, k, n, bf16);
                su += x * proj_w(Bu, Su, H, I, e, k, n, bf16);
            }
            h[n] = orc_tof(orc_fromf((float)(sg / (1.0 + exp(-sg)) *
                                             orc_tof(orc_fromf((float)su, bf16), bf16)), bf16), bf16);
        }
#pragma omp parallel for
        for (int n = 0; n < H; ++n) {
            double s = 0.0;
            for (int k = 0; k < I; ++k) s += h[k] * proj_w(Bd, Sd, I, H, e, k, n, bf16);
            o[n] += s * orc_tof(RW[g], bf16);
        }
    }
    free(h);
}

/* int2_moe/main.cpp:267-291 (the decode driver's check): o[n] = sum_j RW[g] * down(h),
 * h = DT(silu(gate.x) * up.x) in double precision (up not rounded to DT) */
void orc_moe_decode_token_ref(const uint16_t *X, const int *ids, const uint16_t *RW, const uint32_t *Bg,
                              const uint16_t *Sg, const uint32_t *Bu, const uint16_t *Su,
                              const uint32_t *Bd, const uint16_t *Sd, int t, int topk, int H, int I,
                              double *o, int bf16) {
    for (int n = 0; n < H; ++n) o[n] = 0.0;
    float *h = (float *)malloc((size_t)I * sizeof(float));
    for (int j = 0; j < topk; ++j) {
        const int g = t * topk + j, e = ids[g];
#pragma omp parallel for
        for (int n = 0; n < I; ++n) {
            double sg = 0.0, su = 0.0;
            for (int k = 0; k < H; ++k) {
                const double x = orc_tof(X[(size_t)t * H + k], bf16);
                sg += x * proj_w(Bg, Sg, H, I, e, k, n, bf16);
                su += x * proj_w(Bu, Su, H, I, e, k, n, bf16);
            }
            h[n] = orc_tof(orc_fromf((float)(sg / (1.0 + exp(-sg)) * su), bf16), bf16);
        }
#pragma omp parallel for
        for (int n = 0; n < H; ++n) {
            double s = 0.0;
            for (int k = 0; k < I; ++k) s += h[k] * proj_w(Bd, Sd, I, H, e, k, n, bf16);
            o[n] += s * orc_tof(RW[g], bf16);
        }
    }
    free(h);
}
