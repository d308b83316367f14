// Test infrastructure, not product code.  The reference has no host gold for the
// Walsh-Hadamard pre-transform, so this file runs the reference's own OpenCL C
// kernel, hadamard/hadamard_fwht.cl:62-115, on the CPU: the .cl source is
// compiled as C++ under a small OpenCL-C stand-in, and each work-group is executed
// by an OpenMP team of HB/8 threads (one per work-item) whose barriers are
// `omp barrier`; __local arrays become function statics shared by the team.
// One instantiation per (HB, dtype) because both are -D compile options of the .cl.
#include <omp.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace ocl_emu {
typedef unsigned short ushort;
typedef unsigned int uint;
typedef _Float16 half;
static size_t g_group = 0;  // get_group_id(0) of the work-group being emulated
inline size_t get_local_id(int) { return (size_t)omp_get_thread_num(); }
inline size_t get_group_id(int) { return g_group; }
inline half as_half(ushort h) { half x; std::memcpy(&x, &h, 2); return x; }
inline float as_float(uint u) { float f; std::memcpy(&f, &u, 4); return f; }
inline float convert_float(half h) { return (float)h; }
inline half convert_half(float f) { return (half)f; }  // RTE, as OpenCL's default
inline ushort as_ushort(half h) { ushort u; std::memcpy(&u, &h, 2); return u; }
// round to nearest even, NaN quieted (the conversion the .cl names for bf16)
inline ushort intel_convert_bfloat16_as_ushort(float f) {
    uint u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (ushort)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (ushort)(u >> 16);
}
}  // namespace ocl_emu

#define __kernel
#define __global
#define __local static
#define CLK_LOCAL_MEM_FENCE 0
#define barrier(x) _Pragma("omp barrier")
#define reqd_work_group_size(a, b, c) unused

typedef void (*fwht_fn)(const unsigned short *, const char *, unsigned short *, int, int);

#pragma GCC diagnostic push
#pragma GCC diagnostic ignored "-Wunknown-pragmas"
#pragma GCC diagnostic ignored "-Wattributes"

#define HB 256
namespace fp16_256 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 512
namespace fp16_512 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 1024
namespace fp16_1024 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 2048
namespace fp16_2048 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 4096
namespace fp16_4096 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT

#define BF16
#define HB 256
namespace bf16_256 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 512
namespace bf16_512 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 1024
namespace bf16_1024 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 2048
namespace bf16_2048 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#undef HB
#undef LOG2_HB
#undef SCALE
#undef WG
#undef NP8
#undef REM
#undef LOAD_F
#undef STORE_DT
#define HB 4096
namespace bf16_4096 { using namespace ocl_emu;
#include "hadamard/hadamard_fwht.cl"
}
#pragma GCC diagnostic pop

extern "C" {
// y[rows, K] = H_HB(signs * x) / sqrt(HB) per HB block, exactly as the reference
// kernel computes it.  Returns 0 on success, -1 for an unsupported HB or K % HB.
int ref_hadamard_fwht(const unsigned short *x, const signed char *signs, unsigned short *y,
                      int rows, int K, int HBv, int use_signs, int bf16) {
    fwht_fn f = nullptr;
    switch (HBv) {
    case 256: f = bf16 ? bf16_256::hadamard_fwht : fp16_256::hadamard_fwht; break;
    case 512: f = bf16 ? bf16_512::hadamard_fwht : fp16_512::hadamard_fwht; break;
    case 1024: f = bf16 ? bf16_1024::hadamard_fwht : fp16_1024::hadamard_fwht; break;
    case 2048: f = bf16 ? bf16_2048::hadamard_fwht : fp16_2048::hadamard_fwht; break;
    case 4096: f = bf16 ? bf16_4096::hadamard_fwht : fp16_4096::hadamard_fwht; break;
    default: return -1;
    }
    if (K % HBv) return -1;
    const int wg = HBv / 8;
    const size_t groups = (size_t)rows * (size_t)(K / HBv);
    omp_set_dynamic(0);
    int bad = 0;
    for (size_t g = 0; g < groups; ++g) {
        ocl_emu::g_group = g;
#pragma omp parallel num_threads(wg)
        {
            if (omp_get_num_threads() != wg) {
#pragma omp atomic write
                bad = 1;
            } else {
                f(x, (const char *)signs, y, K, use_signs);
            }
        }
        if (bad) return -2;
    }
    return 0;
}
}
