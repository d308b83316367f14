#!/usr/bin/env python3
"""Generate the golden fixtures in this directory from the REFERENCE's own code.

The outputs come from oracle/_ref/libternocl_ref.so, i.e. the reference drivers'
host gold (compute_gold / epilogue_ref / compute_scale_a / to_sel_layout), its BITCOS
packer and decoder (common/bitcos.hpp), its Hadamard kernel source run on the CPU
(hadamard/hadamard_fwht.cl) and the MoE driver's expert-weight decode and generator
(int2_moe/prefill.cpp Proj::w, fill_proj).  It needs oracle/_ref built from the reference tree
(`make -C oracle`), so it runs where the reference sources exist; the .npz fixtures
it writes are committed and pin the oracle everywhere else.

  python tests/golden/make_golden.py [int2 int1 int8 bitcos hadamard moe]
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import api  # noqa: E402
from ternocl_b200 import synth  # noqa: E402

BITCOS_THREADS = 4  # the reference packer's output depends on its OpenMP thread count


def int2_cases(R):
    out = {}
    for bf16 in (0, 1):
        for (M, K, N) in [(3, 256, 48), (1, 512, 32), (77, 128, 16)]:
            rng = np.random.default_rng(1000 + M + K + N + bf16)
            A = synth.activations(rng, M, K, bf16)
            B = synth.pack_int2(synth.ternary(rng, K, N))
            S = synth.scales(rng, K, N, bf16)
            acc = R.int2_gold(A, B, S, M, K, N, bf16)
            key = "int2_%s_%d_%d_%d" % ("bf16" if bf16 else "fp16", M, K, N)
            out[key + "_A"], out[key + "_B"], out[key + "_S"], out[key + "_acc"] = A, B, S, acc
            for postop in range(5):
                for of in (0, 1):
                    other, bias = synth.epilogue_operands(rng, postop, of, M, N, bf16)
                    e = R.epilogue(postop, of, acc, other, bias, M, N, bf16)
                    k2 = "%s_epi%d%s" % (key, postop, "f" if of else "")
                    out[k2 + "_out"] = e
                    if other is not None:
                        out[k2 + "_other"] = other
                    if bias is not None:
                        out[k2 + "_bias"] = bias
    return out


def int1_cases(R):
    out = {}
    for bf16 in (0, 1):
        M, K, N = 3, 256, 48
        rng = np.random.default_rng(2000 + bf16)
        A = synth.activations(rng, M, K, bf16)
        Bpc = rng.integers(0, 2 ** 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
        S = synth.scales(rng, K, N, bf16)
        key = "int1_%s" % ("bf16" if bf16 else "fp16")
        out[key + "_A"], out[key + "_Bpc"], out[key + "_S"] = A, Bpc, S
        out[key + "_acc"] = R.int1_gold(A, Bpc, S, M, K, N, bf16)
        out[key + "_sel"] = R.int1_to_sel(Bpc, K, N)
    return out


def int8_cases(R):
    out = {}
    for bf16 in (0, 1):
        M, K, N = 3, 256, 48
        rng = np.random.default_rng(3000 + bf16)
        A = synth.activations(rng, M, K, bf16)
        B = synth.pack_int2(synth.ternary(rng, K, N))
        SB = synth.scales(rng, K, N, bf16)
        SA = R.int8_scale_a(A, M, K, bf16)
        key = "int8_%s" % ("bf16" if bf16 else "fp16")
        out[key + "_A"], out[key + "_B"], out[key + "_SB"] = A, B, SB
        out[key + "_SA"] = SA
        out[key + "_acc"] = R.int8_gold(A, B, SA, SB, M, K, N, bf16)
    return out


def bitcos_cases(R):
    out = {}
    gomp = ctypes.CDLL("libgomp.so.1")
    gomp.omp_set_num_threads(BITCOS_THREADS)
    for z, seed in [(0.35, 7), (0.05, 11), (0.95, 13)]:
        K, N, M = 256, 48, 3
        buf = R.bitcos_random(K, N, z, seed)
        key = "bitcos_z%02d" % int(round(z * 100))
        out[key + "_buf"] = buf
        out[key + "_codes"] = R.bitcos_decode(buf, K, N)
        for ls in (2, 4):
            out[key + "_sr%d" % ls] = R.bitcos_slice_ranks(buf, K, N, ls)
        for bf16 in (0, 1):
            rng = np.random.default_rng(4000 + seed + bf16)
            A = synth.activations(rng, M, K, bf16)
            S = synth.scales(rng, K, N, bf16)
            k2 = key + ("_bf16" if bf16 else "_fp16")
            out[k2 + "_A"], out[k2 + "_S"] = A, S
            out[k2 + "_acc"] = R.bitcos_gold(A, buf, S, M, K, N, bf16)
    out["bitcos_threads"] = np.array([BITCOS_THREADS])
    return out


def hadamard_cases(R):
    out = {}
    for bf16 in (0, 1):
        for HB in (256, 512, 1024, 2048, 4096):
            rows, K = 2, 2 * HB if HB <= 1024 else HB
            rng = np.random.default_rng(5000 + HB + bf16)
            x = synth.activations(rng, rows, K, bf16)
            s = np.where(rng.random(K) < 0.5, -1, 1).astype(np.int8)
            key = "had_%s_%d" % ("bf16" if bf16 else "fp16", HB)
            out[key + "_x"], out[key + "_s"] = x, s
            out[key + "_y"] = R.hadamard(x, s, rows, K, HB, 1, bf16)
            out[key + "_y0"] = R.hadamard(x, s, rows, K, HB, 0, bf16)
    return out


def moe_cases(R):
    # int2_moe/prefill.cpp:56-79: the expert projections' layout ([E, K/16, N] words,
    # [E, K/128, N] scales) through the driver's own Proj::w, on its own generator's output
    # (fill_proj, codes {0, 1, 3}) and on random words (code 2 as well)
    out = {}
    E, K, N = 3, 256, 16
    for bf16 in (0, 1):
        key = "moe_%s" % ("bf16" if bf16 else "fp16")
        B, S = R.moe_fill(E, K, N, 42, bf16)
        rng = np.random.default_rng(6000 + bf16)
        Br = rng.integers(0, 2 ** 32, size=B.shape, dtype=np.uint64).astype(np.uint32)
        out[key + "_B"], out[key + "_S"], out[key + "_Br"] = B, S, Br
        out[key + "_W"] = R.moe_dequant(B, S, E, K, N, bf16)
        out[key + "_Wr"] = R.moe_dequant(Br, S, E, K, N, bf16)
    return out


CASES = [("int2", int2_cases), ("int1", int1_cases), ("int8", int8_cases), ("bitcos", bitcos_cases),
         ("hadamard", hadamard_cases), ("moe", moe_cases)]


def main():
    """Writes every fixture, or only those named on the command line (e.g. `moe`)."""
    if not api.ref_available():
        sys.exit("oracle/_ref not built: run `make -C oracle` where the reference tree exists")
    R = api.Ref
    for name, fn in CASES:
        if len(sys.argv) > 1 and name not in sys.argv[1:]:
            continue
        d = fn(R)
        path = os.path.join(HERE, "golden_%s.npz" % name)
        np.savez_compressed(path, **d)
        print("wrote", path, os.path.getsize(path), "bytes,", len(d), "arrays")


if __name__ == "__main__":
    main()
