"""Deterministic synthetic inputs for the 800h path, shared by the golden-fixture generator (make_golden.py, run once
in a container where the reference package is importable) and by the tests / bench that check against those fixtures.

Everything is numpy: legacy ``RandomState`` streams (stable across numpy versions and machines) rounded to bf16 with
round-to-nearest-even, so the same seed gives the same bytes on the build container and on the GPU box.  bf16 arrays
are carried as their uint16 bit patterns.

Shapes follow the reference's LFM3 constants: 4 KV heads x head_dim 128, 16 query heads (GQA group 4)."""
import hashlib

import numpy as np

HEADS, DIM, QHEADS = 4, 128, 16


def f32_to_bf16(x):
    """float32 array -> bf16 bit patterns (uint16), round to nearest even (torch's .to(torch.bfloat16))."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h):
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal(seed, shape):
    return np.random.RandomState(seed).standard_normal(shape).astype(np.float32)


def digest(a):
    """sha256 of an array's bytes; float NaNs are first replaced by one canonical NaN (payload and sign bits of a NaN
    are not part of the arithmetic being checked)."""
    a = np.ascontiguousarray(a)
    if a.dtype.kind == "f":
        a = np.where(np.isnan(a), a.dtype.type(np.nan), a)
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------- RoPE tables
def rope_tables(max_pos=8192):
    """cos / sin (max_pos, 32) bf16 bits for the 32 rotating frequency pairs of LFM3's full-attention layers (theta
    1e6), the role of tests/test_parity.py:tables in the reference: fp32 position x fp32 inverse frequency, cos / sin
    evaluated in fp64, rounded to fp32 and then to bf16."""
    inv = (np.float32(1.0) / (np.float32(1e6) ** (np.arange(0, 64, 2, dtype=np.float32) / np.float32(128)))).astype(np.float32)
    fr = np.arange(max_pos, dtype=np.float32)[:, None] * inv[None, :32]
    fr = fr.astype(np.float32).astype(np.float64)
    return f32_to_bf16(np.cos(fr).astype(np.float32)), f32_to_bf16(np.sin(fr).astype(np.float32))


# ---------------------------------------------------------------- quantizer inputs
QUANT_KINDS = ("normal", "outlier", "parity", "edge", "wide")


def quant_inputs(kind, M, seed=0):
    """(k, v) bf16 bits of shape (M, 256, 4, 128) for the quantizer.
      normal  : K, V ~ N(0, 1)
      outlier : N(0, 1) with 1 % of the (head, dim) channels scaled x8
      parity  : K = N(0, 1) + 3 N(0, 1) per-channel offset, V = N(0, 1) (the reference parity test's K)
      edge    : constant channels (zero range), all-zero tokens, all-negative channels, tiny values (subnormal fp8
                scales), large values whose ranges reach the top of the fp8 range
      wide    : K and V spanning several binades per channel (x 2^U[-6, 6])"""
    base = 1000 * QUANT_KINDS.index(kind) + seed
    k = normal(base + 1, (M, 256, HEADS, DIM))
    v = normal(base + 2, (M, 256, HEADS, DIM))
    if kind == "outlier":
        rs = np.random.RandomState(base + 3)
        mk = rs.random_sample((HEADS, DIM)) < 0.01
        mv = rs.random_sample((HEADS, DIM)) < 0.01
        mk[0, 5] = mv[1, 77] = True                       # at least one outlier channel each
        k = np.where(mk[None, None], k * 8, k)
        v = np.where(mv[None, None], v * 8, v)
    elif kind == "parity":
        k = k + 3 * normal(base + 3, (1, 1, HEADS, DIM))
    elif kind == "edge":
        k[:, :, 0, :8] = 1.5                              # constant channels -> (hi - lo) / 3 = 0 -> scale 1e-8 path
        k[:, :, 1, 8:16] = 0.0
        v[:, 7] = 0.0                                     # an all-zero token of V
        v[:, 8, :2] = 0.25                                # a constant V row (its Hadamard image is one spike)
        k[:, :, 2] = -np.abs(k[:, :, 2]) - 2.0            # all-negative channels
        k[:, :, 3, :32] *= 1e-3                           # tiny ranges: subnormal fp8 scales
        v[:, 16:32] *= 1e-3
        k[:, :, 3, 32:48] *= 100.0                        # large ranges: scales near the fp8 max (448)
        k[:, :, 3, 48:64] *= 300.0                        # ranges past it: scale byte 0x7f (NaN), codes 0
        v[:, 32:40] *= 200.0                              # V groups past the fp8 range
        v[:, 40:48] *= 50.0                               # V groups near the top of it
    elif kind == "wide":
        rs = np.random.RandomState(base + 3)
        k = k * np.float32(2.0) ** rs.randint(-6, 7, (1, 1, HEADS, DIM)).astype(np.float32)
        v = v * np.float32(2.0) ** rs.randint(-6, 7, (M, 256, 1, 1)).astype(np.float32)
    return f32_to_bf16(k), f32_to_bf16(v)


# ---------------------------------------------------------------- decode parity cases (reference tests/test_parity.py)
QUANT_NS = (50, 383, 384, 700, 1500, 5000)
WINDOW_NS = (3, 10, 200, 259, 260, 1500)


def parity_cases():
    return [(0, n) for n in QUANT_NS] + [(256, n) for n in WINDOW_NS]


def parity_inputs(win, n, B=2, seed=0):
    """Kh, Vh (B, n, 4, 128) bf16 bits (pre-RoPE K, unrotated V) and q (B, 16, 128) bf16 bits, distributed as in the
    reference parity test (tests/test_parity.py:83-87): K = N(0,1) + 3 N(0,1) per-channel offset, V = N(0,1),
    q = 2 N(0,1)."""
    s = seed * 100003 + n * 7 + win
    K = normal(s + 1, (B, n, HEADS, DIM)) + 3 * normal(s + 2, (1, 1, HEADS, DIM))
    V = normal(s + 3, (B, n, HEADS, DIM))
    q = 2 * normal(s + 4, (B, QHEADS, DIM))
    return f32_to_bf16(K), f32_to_bf16(V), f32_to_bf16(q)
