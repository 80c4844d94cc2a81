"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

The reference quotes no dataset for this path; every config is random-init.  Generators use
numpy's PCG64 with an explicit seed that callers record next to their results.

  C0  MXFP4 matvec 4096x7168: nibbles uniform 0..15, E8M0 uniform 119..127, x ~ N(0,1) f32
  C1  BF16 SwiGLU 2048/768: weights bf16 ~ N(0, 0.02), x bf16 ~ N(0, 1), T in {1, 32}
  C2  MXFP4 MoE 7168 / 256+1 experts / 2048, router bf16 N(0,0.02), bias N(0,0.01), 128 tokens
  C3  MXFP8 grouped 128 experts 4096/1536, E4M3 = fp8-cast N(0,1), E8M0 117..123,
      512 tokens x top-8 Zipf(1.1)
  C4  4 x (7168 / 384+1 experts / 2048) stacked decode, B in {1, 8, 64}
"""
from __future__ import annotations

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16).  Inputs are finite."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def bf16_normal(g: np.random.Generator, shape, std: float) -> np.ndarray:
    """bf16 ~ N(0, std) as uint16 bit patterns."""
    return f32_to_bf16_bits((g.standard_normal(shape, dtype=np.float32) * np.float32(std)))


def encode_e4m3fn(v: np.ndarray) -> np.ndarray:
    """Vectorised src/math/mxfp.rs:247-275 encode_e4m3fn_finite (RNE, saturating at 448)."""
    v = np.clip(np.asarray(v, dtype=np.float32), -448.0, 448.0)
    mag = np.abs(v)
    bits = mag.view(np.uint32)  # |v| <= 448: the rounding below cannot overflow 32 bits
    u = np.uint32  # explicit 32-bit constants keep every operation in uint32
    retained = (bits >> u(20)) & u(1)
    rounded = (bits + u((1 << 19) - 1) + retained) & u(0xFFF00000)
    e = (rounded >> u(23)) & u(0xFF)
    exponent = np.where(e > u(120), e - u(120), u(0))
    mantissa = (rounded >> u(20)) & u(7)
    normal = np.minimum((exponent << u(3)) | mantissa, u(0x7E))
    sub = np.rint(mag * np.float32(512.0)).astype(np.uint32)  # rint = ties-to-even
    code = np.where(mag < np.float32(2.0 ** -6), sub, normal)
    code = np.where(mag == 0, np.uint32(0), code)
    neg = np.signbit(v) & (code != 0)
    return (code.astype(np.uint8) | np.where(neg, np.uint8(0x80), np.uint8(0))).astype(np.uint8)


def mxfp4_matrix(g: np.random.Generator, rows: int, cols: int, exp_lo=119, exp_hi=127,
                 group: int = 32):
    """(packed [rows, ceil(cols/2)] uint8, scales [rows, ceil(cols/group)] uint8)."""
    packed = g.integers(0, 256, size=(rows, (cols + 1) // 2), dtype=np.uint8)
    if cols % 2:
        packed[:, -1] &= 0x0F
    scales = g.integers(exp_lo, exp_hi + 1, size=(rows, -(-cols // group)), dtype=np.uint8)
    return packed, scales


def mxfp8_matrix(g: np.random.Generator, rows: int, cols: int, exp_lo=117, exp_hi=123,
                 block_cols: int = 32):
    values = encode_e4m3fn(g.standard_normal((rows, cols), dtype=np.float32))
    scales = g.integers(exp_lo, exp_hi + 1, size=(rows, -(-cols // block_cols)), dtype=np.uint8)
    return values, scales


def normal_f32(g: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return (g.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def normal_bf16_as_f32(g: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    """bf16 ~ N(0, std) values held in f32 (the reference's activations are f32)."""
    return bf16_bits_to_f32(bf16_normal(g, shape, std))


def zipf_routes(g: np.random.Generator, tokens: int, experts: int, top_k: int, s: float = 1.1):
    """Per token `top_k` distinct experts, sequential sampling without replacement with
    popularity 1/rank^s; rank order is a seeded permutation of the expert ids."""
    perm = g.permutation(experts)
    pop = np.empty(experts, dtype=np.float64)
    pop[perm] = 1.0 / np.arange(1, experts + 1, dtype=np.float64) ** s
    ids = np.empty((tokens, top_k), dtype=np.int32)
    for t in range(tokens):
        p = pop.copy()
        for k in range(top_k):
            c = np.cumsum(p)
            e = int(np.searchsorted(c, g.random() * c[-1], side="right"))
            e = min(e, experts - 1)
            ids[t, k] = e
            p[e] = 0.0
    return ids
