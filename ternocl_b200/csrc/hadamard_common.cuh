// Pieces of the blockwise Walsh-Hadamard transform shared by the standalone kernel
// (hadamard.cu) and the BITCOS GEMV that transforms its staged activations
// (gemv_bitcos.cu).  Every radix-2 stage is the exact fp32 pair (a + b, a - b) and the
// stages run in increasing stride order, as in hadamard_fwht (hadamard/hadamard_fwht.cl),
// so any grouping of the stages gives bit-identical results.
#pragma once
#include <cuda_runtime.h>

namespace ternocl {
namespace fwht {

// fp32 scratch index with one pad word per 16 (bank-conflict-free strided access)
__device__ __forceinline__ int pad16(int i) { return i + (i >> 4); }

// the four radix-2 stages over the bits of j, in increasing order
__device__ __forceinline__ void wht16(float v[16]) {
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if ((j & h) == 0) {
                const float a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
}

}  // namespace fwht
}  // namespace ternocl
