"""Seeded synthetic inputs and numpy weight packers.

The distributions follow the benchmark configurations (ternary weights uniform over
{-1, 0, +1}, per-128-group scales uniform in [0.01, 0.05], activations N(0, 1),
epilogue operands N(0, 1)); the packed layouts are the reference's:

* int2: uint32 [K/16, N], code of row 16kp+j at bits 2j..2j+1, codes {0,1,3} =
  {0,+1,-1} (int2_fp16_upcvt/int2_fp16_upcvt.cl:6-9);
* int1: per-column order uint32 [K/32, N], row k at bit (k%32 & 1)*16 + (k%32)/2
  (int1_fp16_upcvt/main.cpp:76), and the device "sel" layout
  (int1_fp16_upcvt/main.cpp:80-92);
* 16-bit tensors are raw fp16 / bf16 bits (uint16), bf16 rounded to nearest even
  (common/dt16.hpp:30-42).
"""
import numpy as np

GS = 128


def to_dt(x, bf16):
    """float array -> fp16 / bf16 raw bits (round to nearest even)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if bf16:
        u = x.view(np.uint32).astype(np.uint64)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        q = ((u >> 16) | 0x40).astype(np.uint16)
        return np.where(nan, q, r).astype(np.uint16)
    return x.astype(np.float16).view(np.uint16)


def from_dt(h, bf16):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    if bf16:
        return (h.astype(np.uint32) << 16).view(np.float32)
    return h.view(np.float16).astype(np.float32)


def ternary(rng, K, N, zero_frac=None):
    """Ternary codes [K, N]: uniform over {-1,0,+1}, or P(0)=zero_frac."""
    if zero_frac is None:
        return rng.integers(-1, 2, size=(K, N), dtype=np.int8)
    nz = rng.random((K, N)) >= zero_frac
    sgn = np.where(rng.random((K, N)) < 0.5, -1, 1)
    return (nz * sgn).astype(np.int8)


def pack_int2(codes):
    """codes [K, N] in {-1,0,+1} -> uint32 [K/16, N]."""
    codes = np.asarray(codes)
    K, N = codes.shape
    c2 = np.where(codes < 0, 3, codes).astype(np.uint32).reshape(K // 16, 16, N)
    out = np.zeros((K // 16, N), np.uint32)
    for j in range(16):
        out |= c2[:, j, :] << np.uint32(2 * j)
    return out


def unpack_int2(B, K, N):
    """uint32 [K/16, N] -> int8 [K, N] via the 2-bit two's complement reading."""
    B = np.asarray(B, np.uint32)
    out = np.empty((K // 16, 16, N), np.int8)
    for j in range(16):
        c = ((B >> np.uint32(2 * j)) & 3).astype(np.int8)
        out[:, j, :] = np.where(c >= 2, c - 4, c)
    return out.reshape(K, N)


def int1_bit_pos(k):
    r = k % 32
    return (r & 1) * 16 + r // 2


def pack_int1(signs):
    """signs [K, N] in {+1,-1} -> per-column order uint32 [K/32, N] (bit 1 = -1)."""
    signs = np.asarray(signs)
    K, N = signs.shape
    neg = (signs < 0).astype(np.uint32).reshape(K // 32, 32, N)
    out = np.zeros((K // 32, N), np.uint32)
    for r in range(32):
        out |= neg[:, r, :] << np.uint32(int1_bit_pos(r))
    return out


def int1_to_sel(Bpc):
    """per-column int1 words [K/32, N] -> device sel layout: word (kp, n0+p) bit j =
    (row 32kp+2p+(j&1), column n0+j/2)."""
    Bpc = np.asarray(Bpc, np.uint32)
    K32, N = Bpc.shape
    blk = Bpc.reshape(K32, N // 16, 16)  # [kp, block, c]
    out = np.zeros((K32, N // 16, 16), np.uint32)
    for p in range(16):
        w = np.zeros((K32, N // 16), np.uint32)
        for c in range(16):
            for h in range(2):
                bit = (blk[:, :, c] >> np.uint32(h * 16 + p)) & 1
                w |= bit << np.uint32(2 * c + h)
        out[:, :, p] = w
    return out.reshape(K32, N)


def scales(rng, K, N, bf16, lo=0.01, hi=0.05):
    return to_dt(rng.uniform(lo, hi, size=(K // GS, N)), bf16)


def activations(rng, M, K, bf16):
    return to_dt(rng.standard_normal((M, K)), bf16)


def epilogue_operands(rng, postop, out_f32, M, N, bf16):
    """(Other, Bias) for the epilogue, N(0,1); None where the epilogue does not read it."""
    other = to_dt(rng.standard_normal((M, N)), bf16) if postop in (1, 2) else None
    bias = None
    if postop == 3:
        b = rng.standard_normal(N).astype(np.float32)
        bias = b if out_f32 else to_dt(b, bf16)
    return other, bias
