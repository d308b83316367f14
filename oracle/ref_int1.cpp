// Test infrastructure, not product code (see ref_int2.cpp).  Exports the int1
// driver's host functions:
//   bit_pos        int1_fp16_upcvt/main.cpp:76
//   to_sel_layout  int1_fp16_upcvt/main.cpp:80-92
//   compute_gold   int1_fp16_upcvt/main.cpp:95-114
#define main ternocl_ref_int1_main
#include "int1_fp16_upcvt/main.cpp"
#undef main

extern "C" {
void ref_int1_gold(const uint16_t *A, const uint32_t *B, const uint16_t *S, float *C, int M,
                   int K, int N) {
    compute_gold(A, B, S, C, M, K, N);
}
void ref_int1_to_sel(const uint32_t *B, uint32_t *O, int K, int N) { to_sel_layout(B, O, K, N); }
int ref_int1_bit_pos(int k) { return bit_pos(k); }
}
