"""Float32 arithmetic with a fixed operation order, shared by definition with the GPU kernels (test infrastructure).

The GPU's verify decode and acceptance kernels (plm-anon_b200/csrc/voronoi.cu, compiled with -fmad=false) and these
numpy functions perform the same IEEE single-precision operations in the same order, so for identical inputs they
produce identical bits. The elementary functions restate plm-anon_b200/csrc/plm_math.h (Cody-Waite reduction with a
degree-7 Taylor polynomial for exp; the atanh series for log); the reductions restate the kernels' thread layout:

  block_sum  1024 threads, thread t accumulates elements t, t + 1024, ... sequentially from 0; each warp of 32
             threads then combines by an xor butterfly (offsets 16, 8, 4, 2, 1); the 32 warp results are combined
             by the same butterfly.
  lane_sum   one warp: lane l accumulates elements l, l + 32, ... sequentially from 0, then the butterfly.
"""

from __future__ import annotations

import numpy as np

F = np.float32

LN2_HI = F(float.fromhex("0x1.62e4p-1"))
LN2_LO = F(float.fromhex("0x1.7f7d1cp-20"))
LOG2E = F(float.fromhex("0x1.715476p+0"))
EXP_MAX_ARG = F(float.fromhex("0x1.62e43p+6"))
EXP_MIN_ARG = F(float.fromhex("-0x1.9fe36ap+6"))
_EXP_COEFFS = [F(float.fromhex(h)) for h in ("0x1.a01a02p-13", "0x1.6c16c2p-10", "0x1.111112p-7", "0x1.555556p-5",
                                              "0x1.555556p-3", "0x1.0p-1")]
_LOG_COEFFS = [F(float.fromhex(h)) for h in ("0x1.745d18p-4", "0x1.c71c72p-4", "0x1.24924ap-3", "0x1.99999ap-3",
                                              "0x1.555556p-2")]
SQRT2 = F(float.fromhex("0x1.6a09e6p+0"))
TWO_P127 = F(2.0 ** 127)
TWO_M126 = F(2.0 ** -126)
TWO_P23 = F(2.0 ** 23)


def f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def exp32(x) -> np.ndarray:
    """plm_expf, elementwise (plm_math.h)."""
    x = f32(x)
    with np.errstate(all="ignore"):
        n = np.rint(x * LOG2E)
        r = (x - n * LN2_HI) - n * LN2_LO
        p = _EXP_COEFFS[0]
        for c in _EXP_COEFFS[1:]:
            p = p * r + c
        p = p * r + F(1.0)
        p = p * r + F(1.0)
        ni = np.clip(np.nan_to_num(n, nan=0.0, posinf=0.0, neginf=0.0), -200, 200).astype(np.int32)
        hi = ni > 127
        p = np.where(hi, p * TWO_P127, p)
        ni = np.where(hi, ni - 127, ni)
        lo = ni < -126
        p = np.where(lo, p * TWO_M126, p)
        ni = np.where(lo, ni + 126, ni)
        ni = np.clip(ni, -126, 127)
        scale = ((ni + 127).astype(np.uint32) << np.uint32(23)).view(np.float32)
        out = f32(p * scale)
        out = np.where(x > EXP_MAX_ARG, F(np.inf), out)
        out = np.where(x < EXP_MIN_ARG, F(0.0), out)
        out = np.where(np.isnan(x), x, out)
    return f32(out)


def log32(x) -> np.ndarray:
    """plm_logf, elementwise (plm_math.h)."""
    x = f32(x)
    with np.errstate(all="ignore"):
        b = x.view(np.uint32)
        sub = (b < np.uint32(0x00800000)) & (x > 0)
        xs = np.where(sub, x * TWO_P23, x)
        b = f32(xs).view(np.uint32)
        e = np.where(sub, -23, 0).astype(np.int32) + ((b >> np.uint32(23)).astype(np.int32) - 127)
        m = ((b & np.uint32(0x007FFFFF)) | np.uint32(0x3F800000)).view(np.float32)
        big = m > SQRT2
        m = np.where(big, m * F(0.5), m)
        e = e + big.astype(np.int32)
        s = (m - F(1.0)) / (m + F(1.0))
        z = s * s
        p = _LOG_COEFFS[0]
        for c in _LOG_COEFFS[1:]:
            p = p * z + c
        p = p * z + F(1.0)
        lm = (F(2.0) * s) * p
        fe = e.astype(np.float32)
        out = fe * LN2_HI + (fe * LN2_LO + lm)
        out = np.where(x == 0, F(-np.inf), out)
        out = np.where(x == np.inf, F(np.inf), out)
        out = np.where(np.isnan(x) | (x < 0), F(np.nan), out)
    return f32(out)


def _butterfly(values: np.ndarray) -> np.ndarray:
    """xor butterfly over the last axis (length 32); every lane ends with the same value, returned as [..., 0]."""
    v = f32(values)
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        v = v + v[..., lanes ^ off]
    return v[..., 0]


def block_sum(values: np.ndarray, threads: int = 1024) -> np.float32:
    """Sum of a 1-D float32 vector in the kernels' block order (see module docstring)."""
    v = f32(values).ravel()
    acc = np.zeros(threads, dtype=np.float32)
    for start in range(0, v.size, threads):
        part = v[start:start + threads]
        acc[: part.size] = acc[: part.size] + part
    warps = _butterfly(acc.reshape(threads // 32, 32))
    padded = np.zeros(32, dtype=np.float32)
    padded[: warps.size] = warps
    return F(_butterfly(padded[None, :])[0])


def _lane_reduce(values: np.ndarray) -> np.float32:
    acc = np.zeros(32, dtype=np.float32)
    for start in range(0, values.size, 32):
        part = values[start:start + 32]
        acc[: part.size] = acc[: part.size] + part
    return F(_butterfly(acc[None, :])[0])


def lane_sum(values: np.ndarray) -> np.float32:
    """Sum in one warp's order: lane l adds elements l, l + 32, ... from 0, then the butterfly."""
    return _lane_reduce(f32(values).ravel())


def orderable_key(x) -> np.ndarray:
    """Monotone uint32 key of float32 values (plm_math.h orderable_key)."""
    b = f32(x).view(np.uint32)
    return np.where(b & np.uint32(0x80000000), ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def condense_key(cost, target) -> np.ndarray:
    """plm/iterate.py:101-102: ordered cost bits with the low 7 bits replaced by the target index."""
    b = f32(cost).view(np.int32)
    ordered = np.where(b >= 0, b, b ^ np.int32(0x7FFFFFFF))
    return ((ordered & np.int32(~0x7F)) | np.asarray(target, dtype=np.int32)).astype(np.int32)


def condensed_cost(key) -> np.ndarray:
    """plm/iterate.py:132-134: the cost carried by a condensed key."""
    key = np.asarray(key, dtype=np.int32)
    carried = key & np.int32(~0x7F)
    return np.where(carried >= 0, carried, carried ^ np.int32(0x7FFFFFFF)).astype(np.int32).view(np.float32)


def round_to_dtype(x, dtype: str) -> np.ndarray:
    """Round float32 values to the model storage dtype and back (bfloat16 round-to-nearest-even, or float16)."""
    x = f32(x)
    if dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype != "bfloat16":
        raise ValueError(dtype)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)) << np.uint64(16)
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(nan, x, out).astype(np.float32)
