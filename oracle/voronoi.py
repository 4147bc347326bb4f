"""Restatement of the Voronoi verify decode and the acceptance rules (test infrastructure).

Follows plm/iterate.py (the ``iterate`` backend of LogitVoronoiAuxiliary, plm/auxiliary.py:17-75) and
plm/decoder.py:71-82 step by step. Where the reference leaves an order unspecified — float atomics in the fit
(iterate.py:146), Triton's reduction order, torch.topk / argsort tie order — this restatement fixes the order the
GPU kernel (plm-anon_b200/csrc/voronoi.cu) uses, and does its float32 arithmetic with ``oracle.exact``, so that for
identical fp32 logits and cost table both produce the same bits:

  shortlist  the top ``top_m`` logits ordered by (value descending, index ascending); on the tile-max path of
             iterate.py:248-273 ties at the boundary are resolved by torch.topk, here by lower index;
  quota      largest remainder, equal remainders ranked by shortlist position (iterate.py:214-223);
  sums       vocabulary-wide sums are partitioned like the GPU's cluster of CLUSTER ranks: each rank's contiguous
             slice is summed with ``exact.block_sum`` over THREADS threads and the slice sums added in rank order;
             ``exact.lane_sum`` for 128- and 64-element sums; the shortlist softmax in k order; the fit's
             per-target load per rank as a ``lane_sum`` over the target's entries (owned items ascending), the
             rank partials added in rank order — instead of float atomics.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .exact import (F, _butterfly, block_sum, condense_key, condensed_cost, exp32, f32, lane_sum, log32, orderable_key,
                    round_to_dtype)

# The GPU decodes a verify row with a cluster of CLUSTER CTAs of THREADS threads (csrc/verify.h).
CLUSTER = 8
THREADS = 256

# plm/iterate.py:21-25 and the defaults of Voronoi.prior / fit / assign (iterate.py:286, 292-294, 322-324)
STEP_LIMIT = 0.25
LOAD_FLOOR = 1e-2
BLOCKED = 1e3
PRIOR_WEIGHT = 0.1
EPSILON = 0.15
REFOCUS = 0.35
ENDPOINT = 0.0087
RELAX = 1.9


@dataclass
class VoronoiConfig:
    """The scheme fields of plm/auxiliary.py:18-20 (LogitVoronoiAuxiliary.__init__)."""
    top_m: int = 128
    shortlist: int = 8
    rounds: int = 2
    sweeps: int = 12


@dataclass
class Decoded:
    token: int
    tokens: np.ndarray   # [top_m] shortlist token ids
    counts: np.ndarray   # [top_m] quota
    bias: np.ndarray     # [top_m] fitted factors
    sigma: int           # shortlist index of the decoded token
    maximum: np.float32
    total: np.float32
    normaliser: np.float32
    unit: np.float32


def _slices(n: int):
    length = -(-n // CLUSTER)
    return [(min(n, q * length), min(n, (q + 1) * length)) for q in range(CLUSTER)]


def partitioned_sum(values: np.ndarray) -> np.float32:
    """Slice sums in the 256-thread block order, added in rank order (the GPU cluster's vocabulary-wide sums)."""
    total = F(0.0)
    for lo, hi in _slices(values.size):
        total = F(total + block_sum(values[lo:hi], threads=THREADS))
    return total


def row_stats(row: np.ndarray):
    """Maximum, sum of exp(x - max) and normaliser max + log(sum) of one row (iterate.py:54-80 / 176-192)."""
    row = f32(row)
    m = F(row.max())
    total = partitioned_sum(exp32(row - m))
    return m, total, F(m + log32(total))


def shortlist(row: np.ndarray, normaliser: np.float32, top_m: int, n_items: int):
    """Top ``top_m`` tokens and their integer quotas summing to ``n_items`` (iterate.py:248-273, 214-223)."""
    row = f32(row)
    keys = orderable_key(row).astype(np.int64)
    order = np.lexsort((np.arange(row.size), -keys))[:top_m]
    tokens = order.astype(np.int64)
    values = row[tokens]
    probability = exp32(values - normaliser)
    psum = lane_sum(probability)
    weights = probability / psum
    exact = weights * F(n_items)
    counts = np.floor(exact).astype(np.int64)
    remaining = n_items - int(counts.sum())
    frac = exact - counts.astype(np.float32)
    rank = np.empty(top_m, dtype=np.int64)
    rank[np.lexsort((np.arange(top_m), -frac.astype(np.float64)))] = np.arange(top_m)
    return tokens, counts + (rank < remaining).astype(np.int64)


def spread(table: np.ndarray, tokens: np.ndarray, dtype: str, sample: int = 64) -> np.float32:
    """Mean over the first ``sample`` items of (max - min) cost among the shortlist (iterate.py:275-284)."""
    ncols = min(sample, table.shape[1])
    head = table[tokens][:, :ncols]
    diff = round_to_dtype(head.max(axis=0) - head.min(axis=0), dtype)
    return F(lane_sum(diff) / F(ncols))


def prior(counts: np.ndarray, unit: np.float32, n_items: int) -> np.ndarray:
    """iterate.py:286-290."""
    share = np.maximum(counts.astype(np.float32) / F(n_items), F(1e-9))
    return f32(np.where(counts > 0, (F(-PRIOR_WEIGHT) * unit) * log32(share), F(BLOCKED) * unit))


def condense(table: np.ndarray, tokens: np.ndarray, offset: np.ndarray, k: int) -> np.ndarray:
    """Each item's ``k`` cheapest targets under cost + offset, packed as in iterate.py:83-107: int32 [k, A]."""
    cost = table[tokens] + f32(offset)[:, None]
    keys = condense_key(cost, np.arange(tokens.size)[:, None])
    return np.sort(keys, axis=0)[:k]


def _rank_loads(weights_by_target: np.ndarray, present: np.ndarray) -> np.ndarray:
    """Per-target load of one rank: [M, owned] weights and whether the item holds the target (a held entry's weight
    can underflow to 0). One warp per target sums the target's entries (owned items ascending) in ``lane_sum`` order;
    the lanes past the last entry add nothing, which the zero padding reproduces exactly."""
    n_targets = weights_by_target.shape[0]
    pos = np.cumsum(present, axis=1) - 1
    longest = int(present.sum(axis=1).max(initial=0))
    packed = np.zeros((n_targets, max(32, -(-longest // 32) * 32)), dtype=np.float32)
    rows, cols = np.nonzero(present)
    packed[rows, pos[rows, cols]] = weights_by_target[rows, cols]
    acc = np.zeros((n_targets, 32), dtype=np.float32)
    for start in range(0, packed.shape[1], 32):
        acc = acc + packed[:, start:start + 32]
    return f32(_butterfly(acc))


def fit(keys: np.ndarray, counts: np.ndarray, offset: np.ndarray, unit: np.float32, iterations: int,
        epsilon: float, relax: float = RELAX, endpoint: float = ENDPOINT, limit: float = STEP_LIMIT) -> np.ndarray:
    """The annealed Sinkhorn fit of iterate.py:110-159 / 292-312 on the condensed problem."""
    k, n_items = keys.shape
    n_targets = counts.size
    anneal = F((endpoint / epsilon) ** (1.0 / max(iterations, 1)))
    share = log32(np.maximum(counts.astype(np.float32), F(1e-9)))
    temperature = F(F(epsilon) * unit)
    bound = F(F(limit) * unit)
    correction = np.zeros(n_targets, dtype=np.float32)
    target = (keys & 0x7F).astype(np.int64)
    base_cost = condensed_cost(keys)
    owned = n_items // CLUSTER
    columns = np.arange(n_items)
    held = np.zeros((n_targets, n_items), dtype=bool)
    for q in range(k):
        held[target[q], columns] = True
    for _ in range(iterations):
        weight = (-(base_cost + correction[target])) / temperature
        e = exp32(weight - weight.max(axis=0))
        wsum = np.zeros(n_items, dtype=np.float32)
        for q in range(k):
            wsum = wsum + e[q]
        e = e / wsum
        dense = np.zeros((n_targets, n_items), dtype=np.float32)
        for q in range(k):
            dense[target[q], columns] = e[q]
        load = np.zeros(n_targets, dtype=np.float32)
        for rank in range(CLUSTER):
            cols = slice(rank * owned, (rank + 1) * owned)
            load = load + _rank_loads(dense[:, cols], held[:, cols])
        step = temperature * (log32(np.maximum(load, F(LOAD_FLOOR))) - share)
        step = np.minimum(np.maximum(step, -bound), bound)
        corrected = correction + F(relax) * step
        correction = f32(np.where(counts > 0, corrected, F(0.0)))
        temperature = F(temperature * anneal)
    return f32(f32(offset) + correction)


def decode_row(row: np.ndarray, table: np.ndarray, cell: int, dtype: str,
               config: VoronoiConfig = VoronoiConfig()) -> Decoded:
    """The token auxiliary cell ``cell`` holds for one row of logits (auxiliary.py:67-75 -> iterate.py:322-342)."""
    n_items = table.shape[1]
    m, total, normaliser = row_stats(row)
    tokens, counts = shortlist(row, normaliser, config.top_m, n_items)
    unit = spread(table, tokens, dtype)
    bias = prior(counts, unit, n_items)
    for index in range(config.rounds):
        offset = bias
        keys = condense(table, tokens, offset, min(config.shortlist, config.top_m))
        bias = fit(keys, counts, offset, unit, config.sweeps, EPSILON if index == 0 else EPSILON * REFOCUS)
    cell = min(max(int(cell), 0), n_items - 1)
    sigma = int(np.argmin(table[tokens, cell] + bias))
    return Decoded(int(tokens[sigma]), tokens, counts, bias, sigma, m, total, normaliser, unit)


def assign_sigma(table: np.ndarray, tokens: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """sigma(a) for every auxiliary item (iterate.py:314-320, 345-346)."""
    return np.argmin(table[tokens] + f32(bias)[:, None], axis=0)


# ---------------------------------------------------------------- acceptance rules (plm/decoder.py:71-82)

def nucleus_accepts(row: np.ndarray, pending: int, nucleus: float) -> bool:
    """Proposal inside the top-``nucleus`` mass; ``nucleus <= 0`` accepts none (exact match)."""
    nucleus = F(nucleus)
    if not nucleus > 0:
        return False
    row = f32(row)
    m, total, _ = row_stats(row)
    probs = exp32(row - m) / total
    own = probs[pending]
    mass = partitioned_sum(np.where(probs > own, probs, F(0.0)))
    return bool((mass < nucleus) or (own >= probs.max()))


def floor_accepts(row: np.ndarray, pending: int, epsilon: float) -> bool:
    """Proposal with probability above ``epsilon``, in the log domain."""
    row = f32(row)
    _, _, normaliser = row_stats(row)
    return bool((row[pending] - normaliser) > log32(F(epsilon)))
