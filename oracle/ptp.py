"""CPU restatement of the PTP scheme (test infrastructure): the gated-LoRA distilled model's auxiliary pieces.

The reference ships a second auxiliary scheme beside the logit-Voronoi one of every PLM: the linear-interpolation
scheme of its gated-LoRA distilled model (plm/auxiliary.py:78-113, plm/gated_lora.py:35-90). A round then differs
from a PLM round in four places, restated here:

  * the auxiliary stream holds uniforms u in [0, 1) (sample_prior, auxiliary.py:92-94) instead of integer cells, and
    rows that are not auxiliary rows carry the value 0 (no masked value; plm/decoder.py:107-108);
  * an auxiliary row's input vector blends the scheme's float32 embedding rows: u scaled to [0, n - 1], the two
    neighbouring rows weighted by the fraction (auxiliary.py:96-102), cast to the model dtype by the caller
    (decoder.py:264-268);
  * the verify decode is an inverse CDF: the row's softmax at temperature 1, its top_k largest probabilities put in
    token-id order and renormalised, and the token of the first bin whose right edge exceeds u (the last edge is
    forced to 1; auxiliary.py:104-113);
  * every projection that has adapters adds ``x A^T B_s^T`` to its shard s of the output on the rows from the first
    gated row on (gated_lora.py:45-57): row 1 in round 0 (decoder.py:298), row k in a steady round (decoder.py:317),
    no row during prefill (decoder.py:381). The shards of a fused projection (q, k, v; gate, up) share one stacked A,
    and each B maps only its own rank slice back (gated_lora.py:81-90).

Only tests/ may import this module.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class PTPScheme:
    embedding: np.ndarray  # [num_embeddings, hidden] float32
    top_k: int = 128


def linear_interpolation_embed(values: np.ndarray, embedding: np.ndarray) -> np.ndarray:
    """[n] uniforms -> [n, hidden] float32 blends of the two embedding rows around u * (rows - 1)."""
    table = np.asarray(embedding, dtype=np.float32)
    last = table.shape[0] - 1
    scaled = np.asarray(values, dtype=np.float32) * np.float32(last)
    below = np.floor(scaled)
    lo = np.clip(below.astype(np.int64), 0, last)
    hi = np.minimum(lo + 1, last)
    frac = (scaled - below).astype(np.float32)[:, None]
    return (table[lo] * (np.float32(1.0) - frac) + table[hi] * frac).astype(np.float32)


def icdf_probabilities(logits_row: np.ndarray, top_k: int) -> tuple[np.ndarray, np.ndarray]:
    """(token ids ascending, right bin edges) of a row's top_k probabilities, renormalised."""
    x = np.asarray(logits_row, dtype=np.float32)
    e = np.exp(x - x.max(), dtype=np.float32)
    p = (e / e.sum(dtype=np.float32)).astype(np.float32)
    ids = np.sort(np.argsort(-p, kind="stable")[:top_k])
    chosen = p[ids]
    # the running sum in double, each edge rounded to float32 (torch's CPU cumsum of a float32 row)
    edges = np.cumsum((chosen / chosen.sum(dtype=np.float32)).astype(np.float64)).astype(np.float32)
    edges[-1] = np.float32(1.0)
    return ids.astype(np.int64), edges


def icdf_decode_row(logits_row: np.ndarray, u: float, top_k: int) -> int:
    """The token whose bin holds u (the first right edge above u)."""
    ids, edges = icdf_probabilities(logits_row, top_k)
    return int(ids[int(np.argmax(edges > np.float32(u)))])


@dataclass
class Adapter:
    """One projection's adapters: the stacked down-projection [shards * rank, in] and one up-projection
    [shard_out, rank] per output shard, in the projection's own shard order."""
    lora_a: torch.Tensor
    lora_bs: list


def gated_projection(x: torch.Tensor, weight: torch.Tensor, adapter: Adapter | None, rows_from: int | None,
                     rnd, mm) -> torch.Tensor:
    """``x W^T`` on every row, rounded by ``rnd``; rows from ``rows_from`` on add each shard's ``(x A_s^T) B_s^T``:
    the product ``x A^T`` is rounded once, and each shard's correction is added to the rounded base output before
    one more rounding (an in-place multiply-add into the output)."""
    out = rnd(mm(x, weight.T))
    if adapter is None or rows_from is None or rows_from >= x.shape[0]:
        return out
    hidden = rnd(mm(x[rows_from:], adapter.lora_a.T))
    rank = hidden.shape[1] // len(adapter.lora_bs)
    col = 0
    for s, up in enumerate(adapter.lora_bs):
        width = up.shape[0]
        correction = mm(hidden[:, s * rank:(s + 1) * rank], up.T)
        out[rows_from:, col:col + width] = rnd(out[rows_from:, col:col + width] + correction)
        col += width
    return out
