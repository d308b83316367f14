"""Pin the oracle (oracle/oracle.c, the C restatement) against the reference's own
code: the committed golden fixtures (made by tests/golden/make_golden.py from
oracle/_ref, i.e. the reference host gold, BITCOS packer, Hadamard kernel source and
MoE expert-weight decode) and, where oracle/_ref is built, fresh random cases, bit for
bit; the MoE token references, which the reference runs inline in its drivers, against
a numpy recomputation over the pinned decode to 1e-9 (double sums in another order)."""
import ctypes
import os

import numpy as np
import pytest

from oracle import api as orc
from ternocl_b200 import synth

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, "golden_%s.npz" % name))


def same_bits(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_int2_gold_and_epilogues():
    d = load("int2")
    n = 0
    for key in d.files:
        if not key.endswith("_acc"):
            continue
        base = key[:-4]
        _, dt, M, K, N = base.split("_")
        M, K, N, bf16 = int(M), int(K), int(N), int(dt == "bf16")
        acc = orc.int2_gold(d[base + "_A"], d[base + "_B"], d[base + "_S"], M, K, N, bf16)
        assert same_bits(acc, d[key]), base
        for postop in range(5):
            for of in (0, 1):
                k2 = "%s_epi%d%s" % (base, postop, "f" if of else "")
                other = d[k2 + "_other"] if k2 + "_other" in d.files else None
                bias = d[k2 + "_bias"] if k2 + "_bias" in d.files else None
                out = orc.epilogue(postop, of, d[key], other, bias, M, N, bf16)
                assert same_bits(out, d[k2 + "_out"]), k2
                n += 1
    assert n == 6 * 10


def test_int1_gold_and_sel_layout():
    d = load("int1")
    for dt in ("fp16", "bf16"):
        bf16 = int(dt == "bf16")
        k = "int1_" + dt
        M, K, N = 3, 256, 48
        assert same_bits(orc.int1_gold(d[k + "_A"], d[k + "_Bpc"], d[k + "_S"], M, K, N, bf16), d[k + "_acc"])
        assert same_bits(orc.int1_to_sel(d[k + "_Bpc"], K, N), d[k + "_sel"])
        assert same_bits(synth.int1_to_sel(d[k + "_Bpc"]), d[k + "_sel"])


def test_int8_scale_and_gold():
    d = load("int8")
    for dt in ("fp16", "bf16"):
        bf16 = int(dt == "bf16")
        k = "int8_" + dt
        M, K, N = 3, 256, 48
        SA = orc.int8_scale_a(d[k + "_A"], M, K, bf16)
        assert same_bits(SA[:, :M], d[k + "_SA"][:, :M])
        acc = orc.int8_gold(d[k + "_A"], d[k + "_B"], d[k + "_SA"], d[k + "_SB"], M, K, N, bf16)
        assert same_bits(acc, d[k + "_acc"])


def test_bitcos_decode_gold_slice_ranks():
    d = load("bitcos")
    K, N, M = 256, 48, 3
    for z in ("z35", "z05", "z95"):
        k = "bitcos_" + z
        buf = d[k + "_buf"]
        assert orc.orc().orc_bitcos_words(buf.ctypes.data_as(ctypes.c_void_p), K, N) == buf.size
        assert same_bits(orc.bitcos_decode(buf, K, N), d[k + "_codes"])
        for ls in (2, 4):
            assert same_bits(orc.bitcos_slice_ranks(buf, K, N, ls), d[k + "_sr%d" % ls])
        for dt in ("fp16", "bf16"):
            k2 = "%s_%s" % (k, dt)
            acc = orc.bitcos_gold(d[k2 + "_A"], buf, d[k2 + "_S"], M, K, N, int(dt == "bf16"))
            assert same_bits(acc, d[k2 + "_acc"])


def test_hadamard_matches_reference_kernel():
    d = load("hadamard")
    for dt in ("fp16", "bf16"):
        for HB in (256, 512, 1024, 2048, 4096):
            k = "had_%s_%d" % (dt, HB)
            x, s = d[k + "_x"], d[k + "_s"]
            rows, K = x.shape
            bf16 = int(dt == "bf16")
            assert same_bits(orc.hadamard(x, s, rows, K, HB, 1, bf16), d[k + "_y"]), k
            assert same_bits(orc.hadamard(x, s, rows, K, HB, 0, bf16), d[k + "_y0"]), k


@pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref (reference build) not present")
@pytest.mark.parametrize("bf16", [0, 1])
def test_random_cases_vs_reference_build(bf16):
    rng = np.random.default_rng(77 + bf16)
    M, K, N = 5, 1024, 96
    A = synth.activations(rng, M, K, bf16)
    B = synth.pack_int2(synth.ternary(rng, K, N))
    S = synth.scales(rng, K, N, bf16)
    assert same_bits(orc.int2_gold(A, B, S, M, K, N, bf16), orc.Ref.int2_gold(A, B, S, M, K, N, bf16))
    Bpc = rng.integers(0, 2 ** 32, size=(K // 32, N), dtype=np.uint64).astype(np.uint32)
    assert same_bits(orc.int1_gold(A, Bpc, S, M, K, N, bf16), orc.Ref.int1_gold(A, Bpc, S, M, K, N, bf16))
    Af, SA = orc.int8_fake_quant(A, M, K, 0.6, bf16)
    assert same_bits(orc.int8_scale_a(Af, M, K, bf16)[:, :M], orc.Ref.int8_scale_a(Af, M, K, bf16)[:, :M])
    assert same_bits(orc.int8_gold(Af, B, SA, S, M, K, N, bf16), orc.Ref.int8_gold(Af, B, SA, S, M, K, N, bf16))
    buf = orc.Ref.bitcos_random(K, N, 0.4, 3)
    assert same_bits(orc.bitcos_gold(A, buf, S, M, K, N, bf16), orc.Ref.bitcos_gold(A, buf, S, M, K, N, bf16))


def test_moe_expert_weight_decode():
    # int2_moe/prefill.cpp:56-66 (Proj::w): the [E, K/16, N] / [E, K/128, N] expert layout
    # that the MoE token reference and the grouped kernels read
    d = load("moe")
    for bf16 in (0, 1):
        k = "moe_%s" % ("bf16" if bf16 else "fp16")
        B, S, Br = d[k + "_B"], d[k + "_S"], d[k + "_Br"]
        E, K, N = B.shape[0], B.shape[1] * 16, B.shape[2]
        assert same_bits(orc.moe_dequant(B, S, E, K, N, bf16), d[k + "_W"]), k
        assert same_bits(orc.moe_dequant(Br, S, E, K, N, bf16), d[k + "_Wr"]), k
        # the fixture holds the driver's generator output: codes {0, 1, 3} only
        codes = np.stack([(B >> (2 * j)) & 3 for j in range(16)])
        assert set(np.unique(codes).tolist()) == {0, 1, 3}
        # the per-expert reading of the test generator (synth) agrees with Proj::w
        W = d[k + "_Wr"]
        for e in range(E):
            Se = np.repeat(synth.from_dt(S[e], bf16), 128, axis=0)
            assert same_bits((synth.unpack_int2(Br[e], K, N) * Se).astype(np.float32), W[e]), (k, e)


@pytest.mark.parametrize("decode", [False, True], ids=["prefill", "decode"])
@pytest.mark.parametrize("bf16", [0, 1])
def test_moe_token_ref_matches_its_parts(bf16, decode):
    # the token checks of int2_moe/prefill.cpp:291-310 and int2_moe/main.cpp:267-291,
    # recomputed in numpy on top of the pinned expert decode: h = DT(silu(x.Wg) * DT(x.Wu))
    # per routed expert (the decode driver does not round x.Wu to DT), o = sum over the
    # token's experts of RW[g] * (h . Wd), all sums in double
    rng = np.random.default_rng(90 + bf16)
    T, topk, E, H, I = 3, 2, 4, 256, 128
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(T)]).reshape(-1).astype(np.int32)
    X = synth.activations(rng, T, H, bf16)

    def proj(K, N):
        B = rng.integers(0, 2 ** 32, size=(E, K // 16, N), dtype=np.uint64).astype(np.uint32)
        return B, np.stack([synth.scales(rng, K, N, bf16) for _ in range(E)])

    (Bg, Sg), (Bu, Su), (Bd, Sd) = proj(H, I), proj(H, I), proj(I, H)
    RW = synth.to_dt(rng.uniform(0.05, 1.0, T * topk), bf16)
    Wg = orc.moe_dequant(Bg, Sg, E, H, I, bf16).astype(np.float64)
    Wu = orc.moe_dequant(Bu, Su, E, H, I, bf16).astype(np.float64)
    Wd = orc.moe_dequant(Bd, Sd, E, I, H, bf16).astype(np.float64)
    dt = lambda v: synth.from_dt(synth.to_dt(v, bf16), bf16).astype(np.float64)  # noqa: E731
    for t in range(T):
        x = synth.from_dt(X[t], bf16).astype(np.float64)
        o = np.zeros(H)
        for j in range(topk):
            g = t * topk + j
            e = ids[g]
            sg, su = x @ Wg[e], x @ Wu[e]
            h = dt(sg / (1.0 + np.exp(-sg)) * (su if decode else dt(su)))
            o += (h @ Wd[e]) * float(synth.from_dt(RW[g:g + 1], bf16)[0])
        fn = orc.moe_decode_token_ref if decode else orc.moe_token_ref
        ref = fn(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, t, topk, H, I, bf16)
        np.testing.assert_allclose(ref, o, rtol=1e-9, atol=1e-12 * np.abs(o).max())


@pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref (reference build) not present")
def test_moe_decode_vs_reference_build():
    for bf16 in (0, 1):
        B, S = orc.Ref.moe_fill(5, 384, 48, 7 + bf16, bf16)
        assert same_bits(orc.moe_dequant(B, S, 5, 384, 48, bf16), orc.Ref.moe_dequant(B, S, 5, 384, 48, bf16))


def test_int2_value_matches_code_to_value():
    # int2_fp16_upcvt/main.cpp:76: codes {0,1,2,3} -> {0,1,-2,-1}
    B = np.array([[0b11100100]], np.uint32)  # rows 0..3 = codes 0,1,2,3
    vals = [orc.orc().orc_int2_value(B.ctypes.data_as(ctypes.c_void_p), 1, k, 0) for k in range(4)]
    assert vals == [0, 1, -2, -1]
    assert list(synth.unpack_int2(B.reshape(1, 1), 16, 1)[:4, 0]) == [0, 1, -2, -1]
