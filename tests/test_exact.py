"""The fixed-order float32 arithmetic shared by the GPU verify kernel and the oracle (oracle/exact.py,
plm-anon_b200/csrc/plm_math.h): accuracy of the elementary functions against float64, and the key encodings."""

from __future__ import annotations

import numpy as np

from oracle import exact


def _ulps(got: np.ndarray, ref: np.ndarray) -> np.ndarray:
    spacing = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    return np.abs(got.astype(np.float64) - ref) / spacing


def test_exp_accuracy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.uniform(-87, 88, 400_000), rng.uniform(-1, 1, 200_000),
                        rng.uniform(-20, 0, 200_000)]).astype(np.float32)
    assert _ulps(exact.exp32(x), np.exp(x.astype(np.float64))).max() <= 2.0


def test_log_accuracy():
    rng = np.random.default_rng(1)
    y = np.concatenate([rng.uniform(1e-9, 1, 200_000), rng.uniform(0.5, 2, 200_000),
                        np.exp(rng.uniform(-80, 80, 200_000))]).astype(np.float32)
    assert _ulps(exact.log32(y), np.log(y.astype(np.float64))).max() <= 3.0


def test_special_values():
    f = np.float32
    assert exact.exp32(f(0)) == 1 and exact.exp32(f(-200)) == 0 and np.isinf(exact.exp32(f(100)))
    assert np.isnan(exact.exp32(f(np.nan)))
    assert exact.log32(f(1)) == 0 and np.isneginf(exact.log32(f(0))) and np.isnan(exact.log32(f(-1)))
    assert np.isinf(exact.log32(f(np.inf)))
    sub = np.float32(1e-40)
    assert abs(float(exact.log32(sub)) - np.log(1e-40)) < 1e-4
    # the softmax maximum: exp of non-positive arguments never exceeds 1
    xs = -np.arange(0, 1e-3, 1e-7).astype(np.float32)
    assert (exact.exp32(xs) <= 1).all()


def test_block_sum_order():
    v = np.ones(50257, dtype=np.float32)
    assert exact.block_sum(v) == 50257
    # the defined order: per-thread sequential sums, then the warp and block butterflies
    rng = np.random.default_rng(2)
    x = rng.standard_normal(3000).astype(np.float32)
    acc = np.zeros(1024, dtype=np.float32)
    for i, value in enumerate(x):
        acc[i % 1024] = np.float32(acc[i % 1024] + value)
    warps = acc.reshape(32, 32)
    for off in (16, 8, 4, 2, 1):
        warps = warps + warps[:, np.arange(32) ^ off]
    w = warps[:, 0].copy()
    for off in (16, 8, 4, 2, 1):
        w = w + w[np.arange(32) ^ off]
    assert exact.block_sum(x) == w[0]
    assert exact.lane_sum(np.arange(128, dtype=np.float32)) == 8128


def test_condense_key_roundtrip_and_order():
    rng = np.random.default_rng(3)
    cost = (rng.standard_normal(10000) * 10).astype(np.float32)
    target = rng.integers(0, 128, 10000)
    key = exact.condense_key(cost, target)
    assert ((key & 0x7F) == target).all()
    back = exact.condensed_cost(key)
    # the low 7 mantissa bits of |cost| are dropped (toward zero for positive, away for negative keys' order)
    assert np.allclose(back, cost, rtol=2 ** -16, atol=0)
    order = np.argsort(key, kind="stable")
    assert (np.diff(back[order]) >= 0).all()


def test_orderable_key_is_monotone():
    x = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], dtype=np.float32)
    k = exact.orderable_key(x).astype(np.int64)
    assert (np.diff(k) > 0).all()
