"""The C ABI library: it loads, exports every function include/ternocl.h declares,
and validates arguments on the host (no GPU needed for these calls)."""
import ctypes
import os

import numpy as np
import pytest

from ternocl_b200 import _lib, synth


def test_library_exports_every_declared_function():
    L = _lib.lib()
    declared = _lib.header_functions()
    assert len(declared) >= 20
    missing = [f for f in declared if not hasattr(L, f)]
    assert not missing, missing
    # the ctypes table covers exactly the header
    assert sorted(_lib.SIGNATURES) == declared


def test_version_and_status_strings():
    L = _lib.lib()
    assert b"sm_100a" in L.ternocl_version()
    for s in range(8):
        assert L.ternocl_status_string(s)


def test_shape_and_argument_checks_without_gpu():
    L = _lib.lib()
    p = ctypes.c_void_p(64)  # never dereferenced: the checks fail before any device work
    # N % 16 != 0 and K % 128 != 0 (int2_fp16_upcvt/main.cpp:159)
    assert L.ternocl_int2_upcvt(p, p, p, p, None, None, 1, 40, 128, 0, 0, 0, 0, None, 0, None) == 1
    assert L.ternocl_int2_upcvt(p, p, p, p, None, None, 1, 48, 100, 0, 0, 0, 0, None, 0, None) == 1
    # bad dtype / postop / algo
    assert L.ternocl_int2_upcvt(p, p, p, p, None, None, 1, 48, 128, 2, 0, 0, 0, None, 0, None) == 2
    assert L.ternocl_int2_upcvt(p, p, p, p, None, None, 1, 48, 128, 0, 5, 0, 0, None, 0, None) == 2
    # epilogue operand missing
    assert L.ternocl_int2_upcvt(p, p, p, p, None, None, 1, 48, 128, 0, 1, 0, 0, None, 0, None) == 2
    assert L.ternocl_int2_upcvt(p, p, p, p, None, None, 1, 48, 128, 0, 3, 0, 0, None, 0, None) == 2
    # NULL operands, misaligned pointer
    assert L.ternocl_int2_upcvt(None, p, p, p, None, None, 1, 48, 128, 0, 0, 0, 0, None, 0, None) == 2
    q = ctypes.c_void_p(66)
    assert L.ternocl_int2_upcvt(q, p, p, p, None, None, 1, 48, 128, 0, 0, 0, 0, None, 0, None) == 2
    # workspace sizing is a pure host computation
    assert L.ternocl_gemv_workspace_size(1, 40, 128) == 0
    assert L.ternocl_int8_ldsa(1) == 32 and L.ternocl_int8_ldsa(33) == 64


def test_more_host_checks_without_gpu():
    L = _lib.lib()
    p = ctypes.c_void_p(64)
    # s8 x s2: qmode 0/1 only; quant_a needs K % 128
    assert L.ternocl_int2_int8(p, p, p, p, p, p, None, None, 1, 48, 128, 0, 0, 0, 3, 0, None) == 2
    assert L.ternocl_int8_quant_a(p, p, None, 1, 200, 0, None) == 1
    # BITCOS: K % (64 ls), slice ranks needed for ls > 1
    assert L.ternocl_bitcos_upcvt(p, p, p, p, 3, p, None, None, 1, 48, 256, 0, 0, 0, 0, None) == 1
    assert L.ternocl_bitcos_upcvt(p, p, p, None, 2, p, None, None, 1, 48, 256, 0, 0, 0, 0, None) == 2
    # FWHT: HB a power of two in [256, 4096] dividing K
    assert L.ternocl_hadamard_fwht(p, None, p, 1, 5376, 1024, 0, 0, None) == 1
    assert L.ternocl_hadamard_fwht(p, None, p, 1, 4096, 8192, 0, 0, None) == 1
    # MoE: rows per tile is the GEMM's, no bias epilogue, E range
    assert L.ternocl_moe_route(p, p, p, p, 8, 4, 64, None) == 2
    assert L.ternocl_moe_route(p, p, p, p, 8, 0, 128, None) == 1
    assert L.ternocl_moe_gemm(p, p, p, p, p, None, 8, 48, 128, 4, 0, 3, 0, None) == 2
    assert L.ternocl_moe_combine(p, p, p, p, 2, 50, 8, 0, None) == 1
    # int8 MoE: qmode 0 only, SA on 16 bytes, no bias; gather_q needs G = T * topk
    assert L.ternocl_moe_gemm_i8(p, p, p, p, p, p, p, None, 8, 16, 128, 2, 0, 0, 0, 1, None) == 2
    assert L.ternocl_moe_gemm_i8(p, None, p, ctypes.c_void_p(66), p, p, p, None, 8, 16, 128, 2, 0, 0, 0, 0,
                                 None) == 2
    assert L.ternocl_moe_gemm_i8(p, None, p, p, p, p, p, None, 8, 16, 128, 2, 0, 3, 0, 0, None) == 2
    assert L.ternocl_moe_gather_q(p, p, p, p, p, 3, 7, 128, 2, None) == 1
    # fused Hadamard + BITCOS GEMV: HB in 256..2048 dividing K, aligned signs
    assert L.ternocl_bitcos_upcvt_hadamard(p, p, 1, 2048, p, p, None, 1, p, None, None, 1, 48, 4096, 0, 0, 0,
                                           None) == 1
    assert L.ternocl_bitcos_upcvt_hadamard(p, p, 1, 1024, p, p, None, 1, p, None, None, 1, 48, 5376, 0, 0, 0,
                                           None) == 1
    assert L.ternocl_bitcos_upcvt_hadamard(p, ctypes.c_void_p(72), 1, 256, p, p, None, 1, p, None, None, 1, 48,
                                           5376, 0, 0, 0, None) == 2
    # the dense int8 GEMM copies SA rows in 16-byte units: misaligned SA is refused there
    assert L.ternocl_int2_int8(p, p, ctypes.c_void_p(66), p, p, p, None, None, 256, 48, 128, 0, 0, 0, 0, 2,
                               None) == 2


def test_options():
    L = _lib.lib()
    old = L.ternocl_set_option(1, 1)
    assert L.ternocl_set_option(1, old) == 1
    assert L.ternocl_set_option(2, 100) == -1  # GEMM tile rows: 0, 128 or 256
    assert L.ternocl_set_option(2, 256) == 0 and L.ternocl_set_option(2, 0) == 256
    assert L.ternocl_set_option(99, 1) == -1
    # the BITCOS GEMV choice (9): 0 strip kernel at M <= 8, 1 the K-sliced kernel
    assert L.ternocl_set_option(9, 2) == -1
    assert L.ternocl_set_option(9, 1) == 0 and L.ternocl_set_option(9, 0) == 1
    # removed values and the reserved option answer -1 (6: GEMV_IMPL 0..2, 7: reserved)
    assert L.ternocl_set_option(6, 3) == -1 and L.ternocl_set_option(7, 4) == -1


def test_host_bitcos_packer_roundtrip():
    L = _lib.lib()
    rng = np.random.default_rng(3)
    K, N = 256, 48
    codes = synth.ternary(rng, K, N, zero_frac=0.3)
    n = L.ternocl_bitcos_pack(codes.ctypes.data_as(ctypes.c_void_p), K, N, None, 0)
    buf = np.zeros(n, np.uint32)
    assert L.ternocl_bitcos_pack(codes.ctypes.data_as(ctypes.c_void_p), K, N,
                                 buf.ctypes.data_as(ctypes.c_void_p), n) == n
    from oracle import api as orc
    assert np.array_equal(orc.bitcos_decode(buf, K, N), codes.T)


def test_host_bitcos_random_matches_reference_fixture():
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_bitcos.npz"))
    gomp = ctypes.CDLL("libgomp.so.1")
    gomp.omp_set_num_threads(int(d["bitcos_threads"][0]))
    L = _lib.lib()
    K, N = 256, 48
    for z, seed, key in [(0.35, 7, "z35"), (0.05, 11, "z05"), (0.95, 13, "z95")]:
        ref = d["bitcos_%s_buf" % key]
        out = np.zeros(ref.size, np.uint32)
        n = L.ternocl_bitcos_random(K, N, z, seed, out.ctypes.data_as(ctypes.c_void_p), out.size)
        assert n == ref.size and np.array_equal(out, ref), key
        for ls in (2, 4):
            sr = np.zeros((ls - 1, N), np.uint32)
            assert L.ternocl_bitcos_slice_ranks(out.ctypes.data_as(ctypes.c_void_p), K, N, ls,
                                                sr.ctypes.data_as(ctypes.c_void_p)) == 0
            assert np.array_equal(sr, d["bitcos_%s_sr%d" % (key, ls)])


def test_host_int1_sel_matches_reference_fixture():
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_int1.npz"))
    L = _lib.lib()
    Bpc = d["int1_fp16_Bpc"]
    out = np.zeros_like(Bpc)
    assert L.ternocl_int1_to_sel(Bpc.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
                                 256, 48) == 0
    assert np.array_equal(out, d["int1_fp16_sel"])
