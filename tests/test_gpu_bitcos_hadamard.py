"""Hadamard-transformed BITCOS GEMV (ternocl_bitcos_upcvt_hadamard): the sign flip + FWHT
done while the GEMV stages its activations.  Against the two-kernel pipeline it replaces
(ternocl_hadamard_fwht, then ternocl_bitcos_upcvt) bit for bit when both split K the same
way, and against the oracle (the reference's hadamard_fwht restatement, then the BITCOS
host gold, bitcos_fp16_upcvt/main.cpp:64-86) within the output tolerance."""
import numpy as np
import pytest

from helpers import check_output, dev_any, dev_dt, host_dt
from oracle import api as orc
from ternocl_b200 import synth
from test_gpu_bitcos import dev_words

pytestmark = pytest.mark.gpu


def case(tl, seed, M, K, N, z, bf16):
    rng = np.random.default_rng(seed)
    buf = tl.bitcos_random(K, N, z, seed)
    S = synth.scales(rng, K, N, bf16)
    A = synth.activations(rng, M, K, bf16)
    s = np.where(rng.random(K) < 0.5, -1, 1).astype(np.int8)
    return A, buf, S, s


@pytest.fixture
def split(tl):
    # the plain GEMV on the K-sliced kernel, which the fused one extends (the default at
    # M <= 8, the whole-K strip kernel, sums in another order)
    old = tl.set_option(tl.OPT_GEMV_SPLIT, 0)
    old_impl = tl.set_option(tl.OPT_BITCOS_GEMV, 1)
    yield lambda sk: tl.set_option(tl.OPT_GEMV_SPLIT, sk)
    tl.set_option(tl.OPT_GEMV_SPLIT, old)
    tl.set_option(tl.OPT_BITCOS_GEMV, old_impl)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N,hb,sk", [(1, 5376, 512, 256, 1), (1, 5376, 512, 256, 3), (8, 5376, 272, 256, 7),
                                         (3, 4096, 256, 1024, 4), (1, 4096, 1024, 1024, 2), (5, 2048, 128, 512, 2)])
def test_matches_two_kernels(cuda, tl, split, M, K, N, hb, sk, bf16):
    # sk divides both K/128 and K/hb: the fused and the plain GEMV split K alike
    A, buf, S, s = case(tl, M + K + hb, M, K, N, 0.35, bf16)
    dA, dB, dS, ds = dev_dt(A, bf16), dev_words(buf), dev_dt(S, bf16), dev_any(s)
    split(sk)
    for signs in (ds, None):
        fused = host_dt(tl.bitcos_upcvt_hadamard(dA, dB, dS, hb, signs=signs))
        two = host_dt(tl.bitcos_upcvt(tl.hadamard_fwht(dA, hb, signs=signs), dB, dS))
        assert np.array_equal(fused, two), (M, K, N, hb, sk, signs is not None)
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N,hb", [(1, 5376, 512, 256), (8, 5376, 272, 256), (3, 4096, 256, 1024),
                                      (1, 4096, 1024, 512), (2, 1024, 48, 256)])
def test_strip_kernel_matches_two_kernels(cuda, tl, M, K, N, hb, bf16):
    # M <= 8 on the whole-K strip kernel: each CTA transforms its staged rows once, with
    # the standalone kernel's stages, so the result is the two-kernel pipeline's bit for bit
    assert tl.set_option(tl.OPT_BITCOS_GEMV, 0) in (0, 1)
    A, buf, S, s = case(tl, 7 * M + K + hb, M, K, N, 0.35, bf16)
    dA, dB, dS, ds = dev_dt(A, bf16), dev_words(buf), dev_dt(S, bf16), dev_any(s)
    for signs in (ds, None):
        fused = host_dt(tl.bitcos_upcvt_hadamard(dA, dB, dS, hb, signs=signs))
        two = host_dt(tl.bitcos_upcvt(tl.hadamard_fwht(dA, hb, signs=signs), dB, dS))
        assert np.array_equal(fused, two), (M, K, N, hb, signs is not None)
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("M,K,N,ls", [(1, 5376, 512, 1), (8, 5376, 512, 4), (2, 5376, 2048, 7), (4, 1024, 96, 2)])
def test_vs_oracle(cuda, tl, M, K, N, ls, bf16):
    # C4 shape: K = 5376 transforms with HB = 256 (5376 % 1024 != 0)
    hb = 256
    A, buf, S, s = case(tl, 90 + M + N, M, K, N, 0.35, bf16)
    SR = dev_words(tl.bitcos_slice_ranks(buf, K, N, ls)) if ls > 1 else None
    out = host_dt(tl.bitcos_upcvt_hadamard(dev_dt(A, bf16), dev_words(buf), dev_dt(S, bf16), hb, signs=dev_any(s),
                                           SR=SR, ls=ls))
    y = orc.hadamard(A, s, M, K, hb, 1, bf16)
    gold = orc.epilogue(0, False, orc.bitcos_gold(y, buf, S, M, K, N, bf16), None, None, M, N, bf16)
    check_output(out, gold, bf16, False, "M=%d K=%d N=%d ls=%d" % (M, K, N, ls))


@pytest.mark.parametrize("postop,out_f32", [(1, False), (3, True), (4, False)])
def test_epilogues(cuda, tl, postop, out_f32):
    import torch
    M, K, N, hb = 3, 2048, 512, 1024
    A, buf, S, s = case(tl, 7 + postop, M, K, N, 0.2, 0)
    rng = np.random.default_rng(postop)
    other, bias = synth.epilogue_operands(rng, postop, out_f32, M, N, 0)
    dO = dev_dt(other, 0) if other is not None else None
    dBias = (torch.from_numpy(bias).cuda() if out_f32 else dev_dt(bias, 0)) if bias is not None else None
    out = host_dt(tl.bitcos_upcvt_hadamard(dev_dt(A, 0), dev_words(buf), dev_dt(S, 0), hb, signs=dev_any(s),
                                           postop=postop, out_f32=out_f32, other=dO, bias=dBias))
    y = orc.hadamard(A, s, M, K, hb, 1, 0)
    gold = orc.epilogue(postop, out_f32, orc.bitcos_gold(y, buf, S, M, K, N, 0), other, bias, M, N, 0)
    check_output(out, gold, 0, out_f32, "postop=%d out_f32=%d" % (postop, out_f32))
