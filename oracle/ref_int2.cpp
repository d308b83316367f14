// Test infrastructure, not product code.  Built only into oracle/_ref/ by
// oracle/Makefile.  Includes the reference driver int2_fp16_upcvt/main.cpp as it
// lies under the reference tree (compiled with a compile-only CL/cl.h stand-in,
// its main() renamed and never run) and exports the driver's own host gold:
//   compute_gold   int2_fp16_upcvt/main.cpp:79-98
//   epilogue_ref   common/epilogue.hpp:50-67
//   compare        int2_fp16_upcvt/main.cpp:100-121  (xetla_buff_cmp pass rule)
//   compare_f32    common/epilogue.hpp:70-84
#define main ternocl_ref_int2_main
#include "int2_fp16_upcvt/main.cpp"
#undef main

extern "C" {
void ref_set_bf16(int bf16) { dt_is_bf16() = bf16 != 0; }

void ref_int2_gold(const uint16_t *A, const uint32_t *B, const uint16_t *S, float *C, int M,
                   int K, int N) {
    compute_gold(A, B, S, C, M, K, N);
}

void ref_epilogue(int postop, int out_f32, const float *acc, const uint16_t *other,
                  const unsigned char *bias, unsigned char *out, int M, int N) {
    Epilogue e;
    e.postop = postop;
    e.out_f32 = out_f32 != 0;
    epilogue_ref(e, acc, other, bias, out, M, N);
}

// The reference pass rule on a DT output (returns 1 = every element passes).
int ref_compare_dt(const uint16_t *C, const uint16_t *G, size_t n, int postop, int out_f32) {
    Epilogue e;
    e.postop = postop;
    e.out_f32 = out_f32 != 0;
    return compare(C, G, n, "ref-compare", e.abs_tol(), e.ulp_tol()) ? 1 : 0;
}

int ref_compare_f32(const float *C, const float *G, size_t n) {
    return compare_f32(C, G, n, "ref-compare-f32") ? 1 : 0;
}

uint16_t ref_fromf(float f) { return fromf(f); }
float ref_tof(uint16_t h) { return tof(h); }
}
