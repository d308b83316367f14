"""int8 MoE prefill on the GPU (int2_moe/int2_moe_prefill_int8.cl, qmode 0) vs the oracle,
through the C ABI: gather_q (exact: the int8 rows and their scales in expert order), the
grouped s8 x s2 tcgen05 GEMM (each expert's rows vs the int8 host gold of
int2_via_int2_x_int8_dpas/main.cpp:94-121, and bit for bit against the dense int8 GEMM on
the same rows) and a whole layer (quant_a, gather_q, up, gate with SiLU-mul, quant_a of H,
down, combine) vs the double-precision token reference with the reference driver's int8
criterion, max |err| / max |ref| < 5e-2 (int2_moe/prefill.cpp:313-316)."""
import numpy as np
import pytest

from helpers import check_output, dev_any, dev_dt, dev_u32, host_dt
from oracle import api as orc
from ternocl_b200 import synth
from test_gpu_moe import expert_weights, routing

pytestmark = pytest.mark.gpu


def test_gather_q_exact(cuda, tl):
    rng = np.random.default_rng(31)
    T, topk, E, K = 300, 4, 8, 512
    ids = routing(rng, T, topk, E)
    X = synth.activations(rng, T, K, 0)
    SAt, Xq = tl.int8_quant_a(dev_dt(X, 0))
    _, perm, _ = tl.moe_route(dev_any(ids), E)
    Xsq, SA = tl.moe_gather_q(Xq, SAt, perm, topk)
    src = perm.cpu().numpy() // topk
    G = T * topk
    assert np.array_equal(Xsq.cpu().numpy(), Xq.cpu().numpy()[src])
    assert SA.shape == (K // 128, orc.int8_ldsa(G))
    assert np.array_equal(host_dt(SA)[:, :G], host_dt(SAt)[:, src])


def sub_sa(SA, r0, r1):
    """SA columns r0..r1 as the [K/128, LDSA(r1 - r0)] array of an (r1 - r0)-row problem."""
    out = np.zeros((SA.shape[0], orc.int8_ldsa(r1 - r0)), np.uint16)
    out[:, :r1 - r0] = SA[:, r0:r1]
    return out


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop,out_f32", [(0, False), (1, False), (2, False), (0, True)])
def test_grouped_gemm_i8(cuda, tl, bf16, postop, out_f32):
    rng = np.random.default_rng(40 + postop)
    T, topk, E, K, N = 300, 4, 12, 512, 272
    ids = routing(rng, T, topk, E, skew=True)
    G = ids.size
    B, S = expert_weights(rng, E, K, N, bf16)
    A = synth.activations(rng, G, K, bf16)  # already in expert order
    other = synth.to_dt(rng.standard_normal((G, N)), bf16) if postop in (1, 2) else None
    dA = dev_dt(A, bf16)
    SA, Aq = tl.int8_quant_a(dA)
    meta, _, _ = tl.moe_route(dev_any(ids), E)
    dB, dS = dev_u32(B), dev_dt(S, bf16)
    dO = dev_dt(other, bf16) if other is not None else None
    C = host_dt(tl.moe_gemm_i8(meta, Aq, SA, dB, dS, E, postop=postop, out_f32=out_f32, other=dO))
    m = meta.cpu().numpy()
    SAh = host_dt(SA)
    assert np.array_equal(SAh, orc.int8_scale_a(A, G, K, bf16))
    for e in range(E):
        r0, r1 = int(m[e]), int(m[e + 1])
        if r1 == r0:
            continue
        acc = orc.int8_gold(A[r0:r1], B[e], sub_sa(SAh, r0, r1), S[e], r1 - r0, K, N, bf16)
        gold = orc.epilogue(postop, out_f32, acc, other[r0:r1] if other is not None else None, None, r1 - r0, N,
                            bf16)
        check_output(C[r0:r1], gold, bf16, out_f32, "expert %d" % e)
        # the same rows through the dense int8 GEMM: identical per-row arithmetic
        sa_e = dev_dt(sub_sa(SAh, r0, r1), bf16)
        dense = tl.int2_int8(dA[r0:r1].contiguous(), dB[e], dS[e], sa_e, Aq=Aq[r0:r1].contiguous(), qmode=0,
                             postop=postop, out_f32=out_f32, other=dO[r0:r1].contiguous() if dO is not None else None,
                             algo=tl.ALGO_GEMM)
        assert np.array_equal(host_dt(dense), C[r0:r1]), "expert %d differs from the dense GEMM" % e
    assert tl.device_error() == 0


@pytest.mark.parametrize("T,topk,E", [(1, 1, 4), (5, 2, 64), (700, 8, 256)])
def test_grouped_gemm_i8_sparse_routing(cuda, tl, T, topk, E):
    # most experts empty or with a handful of rows; segments start at every offset mod 8
    rng = np.random.default_rng(T + E)
    K, N = 256, 128
    ids = routing(rng, T, topk, E)
    G = ids.size
    B, S = expert_weights(rng, E, K, N, 0)
    A = synth.activations(rng, G, K, 0)
    SA, Aq = tl.int8_quant_a(dev_dt(A, 0))
    meta, _, _ = tl.moe_route(dev_any(ids), E)
    C = host_dt(tl.moe_gemm_i8(meta, Aq, SA, dev_u32(B), dev_dt(S, 0), E))
    m = meta.cpu().numpy()
    SAh = host_dt(SA)
    for e in range(E):
        r0, r1 = int(m[e]), int(m[e + 1])
        if r1 > r0:
            acc = orc.int8_gold(A[r0:r1], B[e], sub_sa(SAh, r0, r1), S[e], r1 - r0, K, N, 0)
            check_output(C[r0:r1], orc.epilogue(0, False, acc, None, None, r1 - r0, N, 0), 0, False, "expert %d" % e)
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
def test_layer_int8_vs_token_reference(cuda, tl, bf16):
    # prefill.cpp's int8 layer (qmode 0): quant_a(X), gather_q, up, gate (POSTOP 1, Other =
    # up), quant_a(H), down (OUT_F32), combine
    rng = np.random.default_rng(22)
    T, topk, E, H, I = 64, 4, 8, 256, 384
    ids = routing(rng, T, topk, E)
    X = synth.activations(rng, T, H, bf16)
    Bg, Sg = expert_weights(rng, E, H, I, bf16)
    Bu, Su = expert_weights(rng, E, H, I, bf16)
    Bd, Sd = expert_weights(rng, E, I, H, bf16)
    gates = rng.standard_normal((T, topk))
    rw = np.exp(gates) / np.exp(gates).sum(1, keepdims=True)
    RW = synth.to_dt(rw.reshape(-1), bf16)
    dX, dRW = dev_dt(X, bf16), dev_dt(RW, bf16)
    meta, perm, inv = tl.moe_route(dev_any(ids), E)
    SAt, Xq = tl.int8_quant_a(dX)
    Xsq, SA1 = tl.moe_gather_q(Xq, SAt, perm, topk)
    dSu, dSg, dSd = dev_dt(Su, bf16), dev_dt(Sg, bf16), dev_dt(Sd, bf16)
    up = tl.moe_gemm_i8(meta, Xsq, SA1, dev_u32(Bu), dSu, E)
    Hh = tl.moe_gemm_i8(meta, Xsq, SA1, dev_u32(Bg), dSg, E, postop=1, other=up)
    SA2, Hq = tl.int8_quant_a(Hh)
    Y = tl.moe_gemm_i8(meta, Hq, SA2, dev_u32(Bd), dSd, E, out_f32=True)
    O = synth.from_dt(host_dt(tl.moe_combine(Y, inv, dRW, T, topk)), bf16)
    max_err = max_ref = 0.0
    for t in range(0, T, 7):
        ref = orc.moe_token_ref(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, t, topk, H, I, bf16)
        max_ref = max(max_ref, float(np.max(np.abs(ref))))
        max_err = max(max_err, float(np.max(np.abs(O[t] - ref))))
    assert max_err / max_ref < 5e-2, "rel %.3g" % (max_err / max_ref)
    assert tl.device_error() == 0
