"""Seeded synthetic quantized-linear operands with the BASELINE distributions.

Generator `numpy.random.default_rng(seed)`, drawn in the order x, codes,
scales:
  x       ~ N(0, 1), rounded to bf16 (round to nearest even)
  codes   uniform over [0, 2**bits), packed little-endian, low bits first,
          along K into u32 words (docs/core/quantized-inference.md:55-62)
  scales  |N(0, 1)| * 0.02 + 1e-3, rounded to bf16
  biases  -2**(bits-1) * scale (exact in bf16: a power-of-two multiple)
"""
import numpy as np


def bf16_round_bits(a):
    """float32 array -> bf16 bit patterns (uint16), round to nearest even."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def pack_codes(codes, bits):
    """codes uint8 [N, K] -> packed u32 [N, K*bits/32], first code in the low bits."""
    N, K = codes.shape
    per = 32 // bits
    out = np.empty((N, K // per), dtype=np.uint32)
    step = max(1, (1 << 24) // max(K, 1))
    shifts = (np.arange(per, dtype=np.uint32) * np.uint32(bits))
    for r0 in range(0, N, step):
        c = codes[r0:r0 + step].astype(np.uint32).reshape(-1, K // per, per)
        out[r0:r0 + step] = np.bitwise_or.reduce(c << shifts, axis=2)
    return out


def quantized_linear(M, N, K, bits=4, group=64, seed=0):
    """Returns dict with x (bf16 bits [M,K]), w (u32 [N,K/P]), s, b (bf16 bits [N,K/g]), codes (uint8 [N,K])."""
    rng = np.random.default_rng(seed)
    x = bf16_round_bits(rng.standard_normal((M, K), dtype=np.float32))
    codes = rng.integers(0, 1 << bits, size=(N, K), dtype=np.uint8)
    s32 = np.abs(rng.standard_normal((N, K // group), dtype=np.float32)) * np.float32(0.02) + np.float32(1e-3)
    s = bf16_round_bits(s32)
    b = bf16_round_bits(-np.float32(1 << (bits - 1)) * bf16_to_f32(s))
    return {"x": x, "w": pack_codes(codes, bits), "s": s, "b": b, "codes": codes, "M": M, "N": N, "K": K,
            "bits": bits, "group": group}
