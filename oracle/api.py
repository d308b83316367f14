"""ctypes view of the test oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the ternocl_b200 product.

Two libraries:
  * ``orc``: oracle/liboracle.so, the C restatement of the reference host gold
    (oracle/oracle.c, each function cites the reference file:line it follows);
  * ``ref``: oracle/_ref/libternocl_ref.so, the reference's OWN host gold compiled
    from its sources (oracle/ref_*.cpp), present wherever it was built.
Arrays are numpy; 16-bit activations/scales are uint16 raw bits.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORC_PATH = os.path.join(HERE, "liboracle.so")
_REF_PATH = os.path.join(HERE, "_ref", "libternocl_ref.so")

_orc = None
_ref = None


def build():
    """Compile the oracle (and oracle/_ref when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


def orc():
    global _orc
    if _orc is None:
        if not os.path.exists(_ORC_PATH):
            build()
        lib = C.CDLL(_ORC_PATH)
        vp, i, f, d, sz = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_size_t
        sig = {
            "orc_tof": (f, [C.c_uint16, i]),
            "orc_fromf": (C.c_uint16, [f, i]),
            "orc_int2_gold": (None, [vp, vp, vp, vp, i, i, i, i]),
            "orc_int2_value": (i, [vp, i, i, i]),
            "orc_int1_bit_pos": (i, [i]),
            "orc_int1_gold": (None, [vp, vp, vp, vp, i, i, i, i]),
            "orc_int1_to_sel": (None, [vp, vp, i, i]),
            "orc_int8_ldsa": (i, [i]),
            "orc_int8_scale_a": (None, [vp, vp, i, i, i]),
            "orc_int8_quant": (None, [vp, vp, vp, i, i, i]),
            "orc_int8_group_dots": (None, [vp, vp, vp, i, i, i]),
            "orc_int8_gold": (None, [vp, vp, vp, vp, vp, i, i, i, i]),
            "orc_int8_fake_quant": (None, [vp, vp, i, i, f, i]),
            "orc_bitcos_words": (sz, [vp, i, i]),
            "orc_bitcos_decode": (None, [vp, i, i, vp]),
            "orc_bitcos_gold": (None, [vp, vp, vp, vp, i, i, i, i]),
            "orc_bitcos_slice_ranks": (None, [vp, i, i, i, vp]),
            "orc_epilogue": (None, [i, i, vp, vp, vp, vp, i, i, i]),
            "orc_hadamard": (i, [vp, vp, vp, i, i, i, i, i]),
            "orc_moe_route": (None, [vp, i, i, i, vp, vp, vp]),
            "orc_moe_dequant": (None, [vp, vp, i, i, i, vp, i]),
            "orc_moe_token_ref": (None, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, vp, i]),
            "orc_moe_decode_token_ref": (None, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, vp, i]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _orc = lib
    return _orc


def ref_available():
    return os.path.exists(_REF_PATH)


def ref():
    """The reference's own compiled host gold (raises if it was never built)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(_REF_PATH + " (build it where the reference tree exists)")
        lib = C.CDLL(_REF_PATH)
        vp, i, f, d, sz, u64 = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_size_t, C.c_uint64
        sig = {
            "ref_set_bf16": (None, [i]),
            "ref_int2_gold": (None, [vp, vp, vp, vp, i, i, i]),
            "ref_epilogue": (None, [i, i, vp, vp, vp, vp, i, i]),
            "ref_compare_dt": (i, [vp, vp, sz, i, i]),
            "ref_compare_f32": (i, [vp, vp, sz]),
            "ref_fromf": (C.c_uint16, [f]),
            "ref_tof": (f, [C.c_uint16]),
            "ref_int1_gold": (None, [vp, vp, vp, vp, i, i, i]),
            "ref_int1_to_sel": (None, [vp, vp, i, i]),
            "ref_int1_bit_pos": (i, [i]),
            "ref_int8_ldsa": (i, [i]),
            "ref_int8_scale_a": (None, [vp, vp, i, i]),
            "ref_int8_gold": (None, [vp, vp, vp, vp, vp, i, i, i]),
            "ref_bitcos_random": (sz, [i, i, d, u64, vp, sz]),
            "ref_bitcos_slice_ranks": (None, [vp, sz, i, i, i, vp]),
            "ref_bitcos_decode_col": (None, [vp, sz, i, i, i, vp]),
            "ref_bitcos_gold": (None, [vp, vp, sz, vp, vp, i, i, i]),
            "ref_hadamard_fwht": (i, [vp, vp, vp, i, i, i, i, i]),
            "ref_moe_dequant": (None, [vp, vp, i, i, i, vp]),
            "ref_moe_fill": (None, [i, i, i, C.c_uint, vp, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _ref = lib
    return _ref


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------------------- oracle (C restatement)
def tof(h, bf16):
    """DT raw bits -> float32 (vectorised, same bits as orc_tof)."""
    h = np.asarray(h, dtype=np.uint16)
    if bf16:
        return (h.astype(np.uint32) << 16).view(np.float32)
    return h.view(np.float16).astype(np.float32)


def int2_gold(A, B, S, M, K, N, bf16):
    A, B, S = _c(A, np.uint16), _c(B, np.uint32), _c(S, np.uint16)
    Cc = np.empty((M, N), np.float32)
    orc().orc_int2_gold(_p(A), _p(B), _p(S), _p(Cc), M, K, N, int(bf16))
    return Cc


def int1_gold(A, B, S, M, K, N, bf16):
    A, B, S = _c(A, np.uint16), _c(B, np.uint32), _c(S, np.uint16)
    Cc = np.empty((M, N), np.float32)
    orc().orc_int1_gold(_p(A), _p(B), _p(S), _p(Cc), M, K, N, int(bf16))
    return Cc


def int1_to_sel(B, K, N):
    B = _c(B, np.uint32)
    O = np.empty_like(B)
    orc().orc_int1_to_sel(_p(B), _p(O), K, N)
    return O


def int8_ldsa(M):
    return (M + 31) & ~31


def int8_scale_a(A, M, K, bf16):
    A = _c(A, np.uint16)
    SA = np.zeros(((K // 128), int8_ldsa(M)), np.uint16)
    orc().orc_int8_scale_a(_p(A), _p(SA), M, K, int(bf16))
    return SA


def int8_quant(A, SA, M, K, bf16):
    A, SA = _c(A, np.uint16), _c(SA, np.uint16)
    Q = np.empty((M, K), np.int8)
    orc().orc_int8_quant(_p(A), _p(SA), _p(Q), M, K, int(bf16))
    return Q


def int8_group_dots(Q, B, M, K, N):
    Q, B = _c(Q, np.int8), _c(B, np.uint32)
    D = np.empty((M, K // 128, N), np.int32)
    orc().orc_int8_group_dots(_p(Q), _p(B), _p(D), M, K, N)
    return D


def int8_gold(A, B, SA, SB, M, K, N, bf16):
    A, B, SA, SB = _c(A, np.uint16), _c(B, np.uint32), _c(SA, np.uint16), _c(SB, np.uint16)
    Cc = np.empty((M, N), np.float32)
    orc().orc_int8_gold(_p(A), _p(B), _p(SA), _p(SB), _p(Cc), M, K, N, int(bf16))
    return Cc


def int8_fake_quant(A, M, K, offgrid, bf16):
    A = np.array(A, dtype=np.uint16, copy=True, order="C")
    SA = np.zeros(((K // 128), int8_ldsa(M)), np.uint16)
    orc().orc_int8_fake_quant(_p(A), _p(SA), M, K, float(offgrid), int(bf16))
    return A, SA


def bitcos_decode(buf, K, N):
    buf = _c(buf, np.uint32)
    codes = np.empty((N, K), np.int8)
    orc().orc_bitcos_decode(_p(buf), K, N, _p(codes))
    return codes


def bitcos_gold(A, buf, S, M, K, N, bf16):
    A, buf, S = _c(A, np.uint16), _c(buf, np.uint32), _c(S, np.uint16)
    Cc = np.empty((M, N), np.float32)
    orc().orc_bitcos_gold(_p(A), _p(buf), _p(S), _p(Cc), M, K, N, int(bf16))
    return Cc


def bitcos_slice_ranks(buf, K, N, ls):
    buf = _c(buf, np.uint32)
    out = np.zeros((max(ls - 1, 0), N), np.uint32)
    if ls > 1:
        orc().orc_bitcos_slice_ranks(_p(buf), K, N, ls, _p(out))
    return out


def epilogue(postop, out_f32, acc, other, bias, M, N, bf16):
    acc = _c(acc, np.float32)
    other = _c(other, np.uint16) if other is not None else None
    if bias is not None:
        bias = _c(bias, np.float32 if out_f32 else np.uint16)
    out = np.empty((M, N), np.float32 if out_f32 else np.uint16)
    orc().orc_epilogue(int(postop), int(out_f32), _p(acc), _p(other), _p(bias), _p(out), M, N,
                       int(bf16))
    return out


def hadamard(x, signs, rows, K, HB, use_signs, bf16):
    x = _c(x, np.uint16)
    signs = _c(signs, np.int8)
    y = np.empty((rows, K), np.uint16)
    rc = orc().orc_hadamard(_p(x), _p(signs), _p(y), rows, K, HB, int(use_signs), int(bf16))
    if rc != 0:
        raise ValueError("bad HB/K")
    return y


def moe_route(ids, E, rows_per_tile):
    ids = _c(ids, np.int32)
    G = ids.size
    meta = np.zeros(2 * E + 2, np.int32)
    perm = np.zeros(G, np.int32)
    inv = np.zeros(G, np.int32)
    orc().orc_moe_route(_p(ids), G, E, rows_per_tile, _p(meta), _p(perm), _p(inv))
    return meta, perm, inv


def moe_dequant(B, S, E, K, N, bf16):
    """int2_moe/prefill.cpp:56-66: every weight of an expert projection, W [E, K, N] float32."""
    B, S = _c(B, np.uint32), _c(S, np.uint16)
    W = np.empty((E, K, N), np.float32)
    orc().orc_moe_dequant(_p(B), _p(S), E, K, N, _p(W), int(bf16))
    return W


def moe_token_ref(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, t, topk, H, I, bf16):
    args = [_c(X, np.uint16), _c(ids, np.int32), _c(RW, np.uint16), _c(Bg, np.uint32),
            _c(Sg, np.uint16), _c(Bu, np.uint32), _c(Su, np.uint16), _c(Bd, np.uint32),
            _c(Sd, np.uint16)]
    o = np.zeros(H, np.float64)
    orc().orc_moe_token_ref(*[_p(a) for a in args], t, topk, H, I, _p(o), int(bf16))
    return o


def moe_decode_token_ref(X, ids, RW, Bg, Sg, Bu, Su, Bd, Sd, t, topk, H, I, bf16):
    """int2_moe/main.cpp:267-291: the decode layer's output for token t (double precision)."""
    args = [_c(X, np.uint16), _c(ids, np.int32), _c(RW, np.uint16), _c(Bg, np.uint32),
            _c(Sg, np.uint16), _c(Bu, np.uint32), _c(Su, np.uint16), _c(Bd, np.uint32),
            _c(Sd, np.uint16)]
    o = np.zeros(H, np.float64)
    orc().orc_moe_decode_token_ref(*[_p(a) for a in args], t, topk, H, I, _p(o), int(bf16))
    return o


# ----------------------------------------------------------------------------- reference (compiled)
class Ref:
    """Thin numpy wrappers over oracle/_ref (the reference's own code)."""

    @staticmethod
    def int2_gold(A, B, S, M, K, N, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        A, B, S = _c(A, np.uint16), _c(B, np.uint32), _c(S, np.uint16)
        Cc = np.empty((M, N), np.float32)
        r.ref_int2_gold(_p(A), _p(B), _p(S), _p(Cc), M, K, N)
        return Cc

    @staticmethod
    def int1_gold(A, B, S, M, K, N, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        A, B, S = _c(A, np.uint16), _c(B, np.uint32), _c(S, np.uint16)
        Cc = np.empty((M, N), np.float32)
        r.ref_int1_gold(_p(A), _p(B), _p(S), _p(Cc), M, K, N)
        return Cc

    @staticmethod
    def int1_to_sel(B, K, N):
        B = _c(B, np.uint32)
        O = np.empty_like(B)
        ref().ref_int1_to_sel(_p(B), _p(O), K, N)
        return O

    @staticmethod
    def int8_scale_a(A, M, K, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        A = _c(A, np.uint16)
        SA = np.zeros(((K // 128), int8_ldsa(M)), np.uint16)
        r.ref_int8_scale_a(_p(A), _p(SA), M, K)
        return SA

    @staticmethod
    def int8_gold(A, B, SA, SB, M, K, N, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        A, B, SA, SB = _c(A, np.uint16), _c(B, np.uint32), _c(SA, np.uint16), _c(SB, np.uint16)
        Cc = np.empty((M, N), np.float32)
        r.ref_int8_gold(_p(A), _p(B), _p(SA), _p(SB), _p(Cc), M, K, N)
        return Cc

    @staticmethod
    def bitcos_random(K, N, z, seed):
        r = ref()
        n = r.ref_bitcos_random(K, N, float(z), int(seed), None, 0)
        out = np.empty(n, np.uint32)
        r.ref_bitcos_random(K, N, float(z), int(seed), _p(out), n)
        return out

    @staticmethod
    def bitcos_slice_ranks(buf, K, N, ls):
        buf = _c(buf, np.uint32)
        out = np.zeros((max(ls - 1, 0), N), np.uint32)
        if ls > 1:
            ref().ref_bitcos_slice_ranks(_p(buf), buf.size, K, N, ls, _p(out))
        return out

    @staticmethod
    def bitcos_decode(buf, K, N):
        buf = _c(buf, np.uint32)
        codes = np.empty((N, K), np.int8)
        r = ref()
        for n in range(N):
            r.ref_bitcos_decode_col(_p(buf), buf.size, K, N, n, codes[n].ctypes.data_as(C.c_void_p))
        return codes

    @staticmethod
    def bitcos_gold(A, buf, S, M, K, N, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        A, buf, S = _c(A, np.uint16), _c(buf, np.uint32), _c(S, np.uint16)
        Cc = np.empty((M, N), np.float32)
        r.ref_bitcos_gold(_p(A), _p(buf), buf.size, _p(S), _p(Cc), M, K, N)
        return Cc

    @staticmethod
    def moe_dequant(B, S, E, K, N, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        B, S = _c(B, np.uint32), _c(S, np.uint16)
        W = np.empty((E, K, N), np.float32)
        r.ref_moe_dequant(_p(B), _p(S), E, K, N, _p(W))
        return W

    @staticmethod
    def moe_fill(E, K, N, seed, bf16):
        """The driver's generator (std::mt19937(seed), fill_proj): B [E, K/16, N], S [E, K/128, N]."""
        r = ref()
        r.ref_set_bf16(int(bf16))
        B = np.empty((E, K // 16, N), np.uint32)
        S = np.empty((E, K // 128, N), np.uint16)
        r.ref_moe_fill(E, K, N, int(seed), _p(B), _p(S))
        return B, S

    @staticmethod
    def epilogue(postop, out_f32, acc, other, bias, M, N, bf16):
        r = ref()
        r.ref_set_bf16(int(bf16))
        acc = _c(acc, np.float32)
        other = _c(other, np.uint16) if other is not None else None
        if bias is not None:
            bias = _c(bias, np.float32 if out_f32 else np.uint16)
        out = np.empty((M, N), np.float32 if out_f32 else np.uint16)
        r.ref_epilogue(int(postop), int(out_f32), _p(acc), _p(other), _p(bias), _p(out), M, N)
        return out

    @staticmethod
    def hadamard(x, signs, rows, K, HB, use_signs, bf16):
        x = _c(x, np.uint16)
        signs = _c(signs, np.int8)
        y = np.empty((rows, K), np.uint16)
        rc = ref().ref_hadamard_fwht(_p(x), _p(signs), _p(y), rows, K, HB, int(use_signs), int(bf16))
        if rc != 0:
            raise ValueError("ref_hadamard_fwht rc=%d" % rc)
        return y

    @staticmethod
    def compare_dt(Cd, G, postop, out_f32, bf16):
        """The reference's xetla_buff_cmp pass rule (int2_fp16_upcvt/main.cpp:100-121)."""
        r = ref()
        r.ref_set_bf16(int(bf16))
        Cd, G = _c(Cd, np.uint16), _c(G, np.uint16)
        return bool(r.ref_compare_dt(_p(Cd), _p(G), Cd.size, int(postop), int(out_f32)))
