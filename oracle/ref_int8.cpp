// Test infrastructure, not product code (see ref_int2.cpp).  Exports the s8 x s2
// driver's host functions:
//   ldsa             int2_via_int2_x_int8_dpas/main.cpp:79
//   compute_scale_a  int2_via_int2_x_int8_dpas/main.cpp:82-91
//   compute_gold     int2_via_int2_x_int8_dpas/main.cpp:94-121
#define main ternocl_ref_int8_main
#include "int2_via_int2_x_int8_dpas/main.cpp"
#undef main

extern "C" {
int ref_int8_ldsa(int M) { return ldsa(M); }
void ref_int8_scale_a(const uint16_t *A, uint16_t *SA, int M, int K) {
    compute_scale_a(A, SA, M, K);
}
void ref_int8_gold(const uint16_t *A, const uint32_t *B, const uint16_t *SA, const uint16_t *SB,
                   float *C, int M, int K, int N) {
    compute_gold(A, B, SA, SB, C, M, K, N);
}
}
