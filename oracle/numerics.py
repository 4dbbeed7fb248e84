"""Bit-level number formats used by the CPU oracle (TEST INFRASTRUCTURE ONLY).

This package is the checker for the CUDA path, never part of it: only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` may import it.

bf16 tensors are carried as ``np.uint16`` bit patterns and fp8-e4m3fn values as
``np.uint8`` bytes, because numpy has neither type.  The conversions follow the
IEEE rules torch applies on CPU:

* fp32 -> bf16: round to nearest, ties to even (``Tensor.to(torch.bfloat16)``).
* fp32 -> fp8 e4m3fn: round to nearest, ties to even, no infinities, |x| <= 448
  after the caller's clamp (``Tensor.to(torch.float8_e4m3fn)`` as used by
  hybrid_attention/dsv4_correctness.py:51).
"""

from __future__ import annotations

import numpy as np

FP8_E4M3_MAX = 448.0


# ----------------------------------------------------------------------------- bf16
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32 exactly."""
    b = np.asarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest, ties to even); returns uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)).astype(np.uint16)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 -> float32."""
    return bf16_to_f32(f32_to_bf16(x))


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ("bf16" | "f16" | "f32") and widen back."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "f32":
        return x
    raise ValueError(f"unknown dtype {dtype}")


# ----------------------------------------------------------------------------- fp8 e4m3fn
def _e4m3_table() -> np.ndarray:
    codes = np.arange(256, dtype=np.uint32)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    mag = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp.astype(np.float64) - 7))
    val = sign * mag
    val[(exp == 15) & (man == 7)] = np.nan
    return val.astype(np.float32)


E4M3_TO_F32 = _e4m3_table()
# Non-negative finite codes 0x00..0x7E are strictly increasing in value.
_E4M3_POS = E4M3_TO_F32[:0x7F].astype(np.float64)


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    return E4M3_TO_F32[np.asarray(codes, dtype=np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """Round float32 values in [-448, 448] to e4m3fn codes (nearest, ties to even)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    hi = np.searchsorted(_E4M3_POS, a, side="left")
    hi = np.clip(hi, 0, 0x7E)
    lo = np.clip(hi - 1, 0, 0x7E)
    d_hi = np.abs(_E4M3_POS[hi] - a)
    d_lo = np.abs(a - _E4M3_POS[lo])
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & (lo % 2 == 0))
    code = np.where(pick_lo, lo, hi).astype(np.uint8)
    code = np.where(np.signbit(x), code | np.uint8(0x80), code).astype(np.uint8)
    return code


# ----------------------------------------------------------------------------- helpers
def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Widen a stored tensor (bf16 bits / f16 / f32) to float32."""
    if dtype == "bf16":
        return bf16_to_f32(x)
    return np.asarray(x).astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 to the storage form of ``dtype`` (bf16 -> uint16 bits)."""
    if dtype == "bf16":
        return f32_to_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    return np.asarray(x, dtype=np.float32)
