// Test infrastructure, not product code (see ref_int2.cpp).  Exports the BITCOS
// driver's gold and the reference packer/decoder:
//   compute_gold         bitcos_fp16_upcvt/main.cpp:64-86
//   bitcos_random        common/bitcos.hpp:31-78
//   bitcos_slice_ranks   common/bitcos.hpp:81-94
//   bitcos_decode_col    common/bitcos.hpp:97-106
#define main ternocl_ref_bitcos_main
#include "bitcos_fp16_upcvt/main.cpp"
#undef main

static Bitcos wrap(const uint32_t *buf, size_t words, int K, int N) {
    Bitcos b;
    b.K = K;
    b.N = N;
    b.buf.assign(buf, buf + words);
    return b;
}

extern "C" {
// Pack with the reference packer.  Returns the buffer length in words; copies the
// buffer into out when out_cap is large enough.
size_t ref_bitcos_random(int K, int N, double z, uint64_t seed, uint32_t *out, size_t out_cap) {
    const Bitcos b = bitcos_random(K, N, z, seed);
    if (out && out_cap >= b.buf.size()) std::copy(b.buf.begin(), b.buf.end(), out);
    return b.buf.size();
}
void ref_bitcos_slice_ranks(const uint32_t *buf, size_t words, int K, int N, int ls, uint32_t *out) {
    const std::vector<uint32_t> r = bitcos_slice_ranks(wrap(buf, words, K, N), ls);
    std::copy(r.begin(), r.end(), out);
}
void ref_bitcos_decode_col(const uint32_t *buf, size_t words, int K, int N, int n, int8_t *codes) {
    bitcos_decode_col(wrap(buf, words, K, N), n, codes);
}
void ref_bitcos_gold(const uint16_t *A, const uint32_t *buf, size_t words, const uint16_t *S,
                     float *C, int M, int K, int N) {
    compute_gold(A, wrap(buf, words, K, N), S, C, M);
}
}
