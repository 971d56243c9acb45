"""Seeded synthetic inputs for the benchmark configurations (numpy; no datasets involved).

- ``conversion_inputs(n)``: the narrow-float round-trip set: 90% N(0,1) * 2^U(-20,20), 10% drawn
  from specials (both zeros, infinities, quiet and signalling NaNs of both signs, f32 subnormals,
  the max-finite / first-overflow / tie values of E4M3, E5M2 and E2M1, and exact
  round-to-nearest-even ties at every binade of each format), with random signs.
- ``mxfp8_activation(rows, cols)``: bf16 N(0,1) * 2^U(-8,8) per row; every 64th row gets one
  element x100 (the MXFP8 quantise workload is 8192 x 8192).
- ``fp8_operand(rows, cols)``: uniform over all finite E4M3 codes with |x| <= 8.
- ``normal_bf16(rows, cols, std)``: bf16 N(0, std^2).
"""

from __future__ import annotations

import numpy as np

SEED = 0x5EED


def _bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def _format_ties(e: int, m: int, bias: int, max_mag: float) -> list[float]:
    reps = [0.0]
    for ex in range(0, 1 << e):
        for mn in range(1 << m):
            v = (mn * 2.0 ** (1 - bias - m)) if ex == 0 else (((1 << m) + mn) *
                                                               2.0 ** (ex - bias - m))
            if v <= max_mag:
                reps.append(v)
    reps = sorted(set(reps))
    return [(a + b) / 2 for a, b in zip(reps, reps[1:])] + reps


def special_values() -> np.ndarray:
    sp = [0.0, np.inf, np.nan, 448.0, 464.0, 480.0, 57344.0, 61440.0, 6.0, 7.0, 1e38, 3.4e38,
          2.0 ** -9, 2.0 ** -10, 2.0 ** -16, 2.0 ** -17, 0.5, 0.25, 0.75, 2.0 ** -127,
          2.0 ** -126, 1.0, 1.5]
    sp += _format_ties(4, 3, 7, 448.0) + _format_ties(5, 2, 15, 57344.0) + \
        _format_ties(2, 1, 1, 6.0)
    bits = np.array(sp, dtype=np.float32).view(np.uint32)
    extra = np.array([0x7FC00000, 0x7F800001, 0x7FBFFFFF, 0x7FFFFFFF,  # quiet / signalling NaN
                      0x00000001, 0x00400000, 0x007FFFFF, 0x00012345],  # f32 subnormals
                     dtype=np.uint32)
    return np.concatenate([bits, extra]).view(np.float32)


def conversion_inputs(n: int = 1 << 24, seed: int = SEED + 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    n_sp = n // 10
    x = (rng.standard_normal(n - n_sp) * np.exp2(rng.uniform(-20, 20, n - n_sp))).astype(
        np.float32)
    sp = special_values()
    pick = sp[rng.integers(0, sp.size, n_sp)].view(np.uint32)
    pick = pick ^ (rng.integers(0, 2, n_sp, dtype=np.uint32) << 31)  # random sign
    out = np.concatenate([x, pick.view(np.float32)])
    # the specials table itself, both signs, at the front so every one is present
    both = np.concatenate([sp.view(np.uint32), sp.view(np.uint32) ^ np.uint32(0x80000000)])
    out[: both.size] = both.view(np.float32)
    perm = rng.permutation(n - both.size) + both.size
    out[both.size:] = out[perm]
    return out


def mxfp8_activation(rows: int = 8192, cols: int = 8192, seed: int = SEED + 2) -> np.ndarray:
    """bf16 bit patterns [rows, cols]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    x *= np.exp2(rng.uniform(-8, 8, (rows, 1))).astype(np.float32)
    out_rows = np.arange(0, rows, 64)
    x[out_rows, rng.integers(0, cols, out_rows.size)] *= 100.0
    return _bf16(x)


def fp8_operand(rows: int, cols: int, seed: int) -> np.ndarray:
    """E4M3 codes uniform over the finite codes with |x| <= 8 (0x00..0x50 and negatives)."""
    codes = np.array([c for c in range(256) if (c & 0x7F) <= 0x50], dtype=np.uint8)
    rng = np.random.default_rng(seed)
    return codes[rng.integers(0, codes.size, (rows, cols))]


def normal_bf16(rows: int, cols: int, std: float = 1.0, seed: int = SEED + 3) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return _bf16(x)
