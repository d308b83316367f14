/* Test oracle: a plain-C restatement of the reference's host gold.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the ternocl_b200 product links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg do, as the checker.  Every function cites the reference file:line it
 * restates (paths relative to the reference tree).  It is pinned against the
 * reference's own compiled host gold (oracle/_ref, see ref_*.cpp) and against the
 * golden fixtures in tests/golden/.
 *
 * dtype convention: 16-bit activations/scales/outputs are raw uint16 bits, fp16
 * when bf16 == 0, bf16 otherwise (common/dt16.hpp:10-42). */
#ifndef TERNOCL_ORACLE_H
#define TERNOCL_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float orc_tof(uint16_t h, int bf16);
uint16_t orc_fromf(float f, int bf16);

/* int2 upconvert GEMM/GEMV fp32 accumulator (before the epilogue). */
void orc_int2_gold(const uint16_t *A, const uint32_t *B, const uint16_t *S, float *C, int M, int K,
                   int N, int bf16);
/* Decoded int2 weight value {-2,-1,0,1} of row k, column n. */
int orc_int2_value(const uint32_t *B, int N, int k, int n);

/* int1: per-column bit order gold and the device "sel" layout. */
int orc_int1_bit_pos(int k);
void orc_int1_gold(const uint16_t *A, const uint32_t *B, const uint16_t *S, float *C, int M, int K,
                   int N, int bf16);
void orc_int1_to_sel(const uint32_t *B, uint32_t *O, int K, int N);

/* s8 x s2: activation scales, int8 codes, per-group int32 dots, fp32 accumulator. */
int orc_int8_ldsa(int M);
void orc_int8_scale_a(const uint16_t *A, uint16_t *SA, int M, int K, int bf16);
void orc_int8_quant(const uint16_t *A, const uint16_t *SA, int8_t *Q, int M, int K, int bf16);
void orc_int8_group_dots(const int8_t *Q, const uint32_t *B, int32_t *D, int M, int K, int N);
void orc_int8_gold(const uint16_t *A, const uint32_t *B, const uint16_t *SA, const uint16_t *SB,
                   float *C, int M, int K, int N, int bf16);
/* The driver's input conditioning: fake-quantise A onto the int8 grid (optionally
 * `offgrid` LSB away from it) and recompute SA. */
void orc_int8_fake_quant(uint16_t *A, uint16_t *SA, int M, int K, float offgrid, int bf16);

/* BITCOS: decode all columns into codes[n*K + k], gold, slice ranks. */
size_t orc_bitcos_words(const uint32_t *buf, int K, int N);
void orc_bitcos_decode(const uint32_t *buf, int K, int N, int8_t *codes);
void orc_bitcos_gold(const uint16_t *A, const uint32_t *buf, const uint16_t *S, float *C, int M,
                     int K, int N, int bf16);
void orc_bitcos_slice_ranks(const uint32_t *buf, int K, int N, int ls, uint32_t *out);

/* Fused epilogue on the fp32 accumulator + output cast (bias: DT, or fp32 if
 * out_f32; out: DT, or fp32 if out_f32). */
void orc_epilogue(int postop, int out_f32, const float *acc, const uint16_t *other,
                  const void *bias, void *out, int M, int N, int bf16);

/* Sign flip + blockwise normalised FWHT. Returns 0, or -1 for a bad HB / K. */
int orc_hadamard(const uint16_t *x, const int8_t *signs, uint16_t *y, int rows, int K, int HB,
                 int use_signs, int bf16);

/* MoE prefill routing with a stable (ascending g) order inside each expert. */
void orc_moe_route(const int *ids, int G, int E, int rows_per_tile, int *meta, int *perm, int *inv);
/* Every weight of a [E, K/16, N] int2 projection with [E, K/128, N] scales, as floats. */
void orc_moe_dequant(const uint32_t *B, const uint16_t *S, int E, int K, int N, float *W, int bf16);
/* The reference driver's double-precision check of token t's layer output o[H]. */
void orc_moe_token_ref(const uint16_t *X, const int *ids, const uint16_t *RW, const uint32_t *Bg,
                       const uint16_t *Sg, const uint32_t *Bu, const uint16_t *Su,
                       const uint32_t *Bd, const uint16_t *Sd, int t, int topk, int H, int I,
                       double *o, int bf16);
void orc_moe_decode_token_ref(const uint16_t *X, const int *ids, const uint16_t *RW, const uint32_t *Bg,
                              const uint16_t *Sg, const uint32_t *Bu, const uint16_t *Su,
                              const uint32_t *Bd, const uint16_t *Sd, int t, int topk, int H, int I,
                              double *o, int bf16);

#ifdef __cplusplus
}
#endif
#endif
