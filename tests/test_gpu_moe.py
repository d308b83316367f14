"""int2 MoE prefill on the GPU (int2_moe/int2_moe_prefill.cl) vs the oracle, through the
C ABI: routing (exact: meta, perm, inv; rows ascending in g inside an expert), gather
(exact), the grouped tcgen05 GEMM (each expert's rows vs the int2 host gold) and a
whole layer (up, gate with SiLU-mul, down, combine) vs the double-precision token
reference of int2_moe/prefill.cpp:291-310."""
import numpy as np
import pytest

from helpers import MOE_TOL, check_output, dev_any, dev_dt, dev_u32, host_dt, moe_layer_err
from oracle import api as orc
from ternocl_b200 import synth

pytestmark = pytest.mark.gpu


def routing(rng, T, topk, E, skew=False):
    """topk distinct experts per token (uniform, or skewed towards low ids)."""
    if skew:
        p = 1.0 / np.arange(1, E + 1)
        p /= p.sum()
        ids = np.stack([rng.choice(E, topk, replace=False, p=p) for _ in range(T)])
    else:
        ids = np.stack([rng.permutation(E)[:topk] for _ in range(T)])
    return ids.reshape(-1).astype(np.int32)


@pytest.mark.parametrize("T,topk,E,skew", [(4096, 8, 128, False), (1000, 4, 16, True), (37, 2, 64, False),
                                           (1, 1, 4, False), (3000, 8, 256, True)])
def test_route_exact(cuda, tl, T, topk, E, skew):
    rng = np.random.default_rng(T + E)
    ids = routing(rng, T, topk, E, skew)
    meta, perm, inv = tl.moe_route(dev_any(ids), E)
    m0, p0, i0 = orc.moe_route(ids, E, tl.moe_rows_per_tile())
    assert np.array_equal(meta.cpu().numpy(), m0)
    assert np.array_equal(perm.cpu().numpy(), p0)
    assert np.array_equal(inv.cpu().numpy(), i0)
    assert tl.device_error() == 0


def test_gather_exact(cuda, tl):
    rng = np.random.default_rng(3)
    T, topk, E, K = 300, 4, 8, 512
    ids = routing(rng, T, topk, E)
    X = synth.activations(rng, T, K, 0)
    _, perm, _ = tl.moe_route(dev_any(ids), E)
    Xs = host_dt(tl.moe_gather(dev_dt(X, 0), perm, topk))
    assert np.array_equal(Xs, X[perm.cpu().numpy() // topk])


def expert_weights(rng, E, K, N, bf16):
    B = np.stack([synth.pack_int2(synth.ternary(rng, K, N)) for _ in range(E)])
    S = np.stack([synth.scales(rng, K, N, bf16) for _ in range(E)])
    return B, S


@pytest.fixture(params=[(0, 128), (0, 256), (1, 0), (3, 0)], ids=["one_cta_per_tile", "rows256", "persistent", "auto"])
def persistent(request, tl):
    pers, tile = request.param
    old = tl.set_option(tl.OPT_GEMM_PERSISTENT, pers)
    old_tile = tl.set_option(tl.OPT_GEMM_TILE_M, tile)
    yield pers
    tl.set_option(tl.OPT_GEMM_PERSISTENT, old)
    tl.set_option(tl.OPT_GEMM_TILE_M, old_tile)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("postop,out_f32", [(0, False), (1, False), (0, True)])
def test_grouped_gemm(cuda, tl, persistent, bf16, postop, out_f32):
    rng = np.random.default_rng(10 + postop)
    T, topk, E, K, N = 400, 4, 12, 512, 272
    ids = routing(rng, T, topk, E, skew=True)
    G = ids.size
    B, S = expert_weights(rng, E, K, N, bf16)
    A = synth.activations(rng, G, K, bf16)
    other = synth.to_dt(rng.standard_normal((G, N)), bf16) if postop == 1 else None
    meta, perm, inv = tl.moe_route(dev_any(ids), E)
    C = host_dt(tl.moe_gemm(meta, dev_dt(A, bf16), dev_u32(B), dev_dt(S, bf16), E, postop=postop, out_f32=out_f32,
                            other=dev_dt(other, bf16) if other is not None else None))
    m = meta.cpu().numpy()
    for e in range(E):
        r0, r1 = m[e], m[e + 1]
        if r1 == r0:
            continue
        acc = orc.int2_gold(A[r0:r1], B[e], S[e], r1 - r0, K, N, bf16)
        gold = orc.epilogue(postop, out_f32, acc, other[r0:r1] if other is not None else None, None, r1 - r0, N,
                            bf16)
        check_output(C[r0:r1], gold, bf16, out_f32, "expert %d" % e)


@pytest.mark.parametrize("bf16", [0, 1])
def test_grouped_gemm_decode_bit_exact(cuda, tl, persistent, bf16):
    # every routed expert gets the K x K identity as its rows, so its output block is its
    # decoded weight matrix: C[r0 + k, n] = code(k, n) * S[k/128, n] through one non-zero
    # term, exact in fp32.  Compared bit for bit with the expert-weight decode of
    # int2_moe/prefill.cpp:56-66 (Proj::w); random words, so every 2-bit code; expert 3
    # gets no rows
    rng = np.random.default_rng(50 + bf16)
    E, K, N = 6, 256, 144
    used = [0, 1, 2, 4, 5]
    ids = np.repeat(np.array(used, np.int32), K)
    B = rng.integers(0, 1 << 32, size=(E, K // 16, N), dtype=np.uint64).astype(np.uint32)
    S = np.stack([synth.scales(rng, K, N, bf16) for _ in range(E)])
    A = np.tile(synth.to_dt(np.eye(K), bf16), (len(used), 1))
    meta, _, _ = tl.moe_route(dev_any(ids), E)
    C = host_dt(tl.moe_gemm(meta, dev_dt(A, bf16), dev_u32(B), dev_dt(S, bf16), E, out_f32=True))
    W = orc.moe_dequant(B, S, E, K, N, bf16)
    m = meta.cpu().numpy()
    assert m[3] == m[4]
    for e in used:
        r0, r1 = int(m[e]), int(m[e + 1])
        assert r1 - r0 == K
        assert np.array_equal(C[r0:r1].view(np.uint32), W[e].view(np.uint32)), "expert %d" % e
    assert tl.device_error() == 0


@pytest.mark.parametrize("bf16", [0, 1])
def test_layer_vs_token_reference(cuda, tl, persistent, bf16):
    # prefill.cpp's layer: up = gemm(Xs, Bu), H = gemm(Xs, Bg, POSTOP 1, Other = up),
    # Y = gemm(H, Bd, OUT_F32), O = combine(Y)
    import torch
    rng = np.random.default_rng(21)
    T, topk, E, H, I = 64, 4, 8, 256, 384
    ids = routing(rng, T, topk, E)
    G = ids.size
    X = synth.activations(rng, T, H, bf16)
    Bg, Sg = expert_weights(rng, E, H, I, bf16)
    Bu, Su = expert_weights(rng, E, H, I, bf16)
    Bd, Sd = expert_weights(rng, E, I, H, bf16)
    gates = rng.standard_normal((T, topk))
    rw = np.exp(gates) / np.exp(gates).sum(1, keepdims=True)
    RW = synth.to_dt(rw.reshape(-1), bf16)
    dX, dRW = dev_dt(X, bf16), dev_dt(RW, bf16)
    meta, perm, inv = tl.moe_route(dev_any(ids), E)
    Xs = tl.moe_gather(dX, perm, topk)
    up = tl.moe_gemm(meta, Xs, dev_u32(Bu), dev_dt(Su, bf16), E)
    Hh = tl.moe_gemm(meta, Xs, dev_u32(Bg), dev_dt(Sg, bf16), E, postop=1, other=up)
    Y = tl.moe_gemm(meta, Hh, dev_u32(Bd), dev_dt(Sd, bf16), E, out_f32=True)
    O = synth.from_dt(host_dt(tl.moe_combine(Y, inv, dRW, T, topk)), bf16)
    toks = (0, 1, T // 2, T - 1)
    refs = [orc.moe_token_ref(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, t, topk, H, I, bf16) for t in toks]
    e = moe_layer_err(O[list(toks)], refs)
    assert e <= MOE_TOL[bf16], "layer rel err %.3g" % e
    assert tl.device_error() == 0


def test_combine(cuda, tl):
    import torch
    rng = np.random.default_rng(5)
    T, topk, N = 50, 8, 512
    G = T * topk
    Y = rng.standard_normal((G, N)).astype(np.float32)
    inv = rng.permutation(G).astype(np.int32)
    RW = synth.to_dt(rng.random(G), 0)
    O = host_dt(tl.moe_combine(torch.from_numpy(Y).cuda(), dev_any(inv), dev_dt(RW, 0), T, topk))
    w = synth.from_dt(RW, 0).astype(np.float64)
    want = np.zeros((T, N))
    for j in range(topk):
        g = np.arange(T) * topk + j
        want += w[g, None] * Y[inv[g]]
    check_output(O, synth.to_dt(want, 0), 0, False, "combine")


def test_route_rejects_bad_ids(cuda, tl):
    ids = np.array([0, 1, 9, 2], np.int32)  # 9 >= E
    tl.device_error(reset=True)
    tl.moe_route(dev_any(ids), 4)
    import torch
    torch.cuda.synchronize()
    assert tl.device_error() & 2
