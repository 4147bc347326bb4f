"""The round's layout tables (same interface as the reference's plm/mask.py).

A round packs ``k`` verify rows, which check last round's chain causally, and ``k`` proposal blocks, each written as
though the prefix it assumes were confirmed, so blocks never see each other. The attention kernel evaluates the
mask from ``depth`` and ``own_start``: key kv is visible to query row r (logical index offset + r) iff
``kv - offset <= depth[r]`` or (``kv - offset >= own_start[r]`` and ``kv <= offset + r``) — plm/mask.py:23-29.
"""

from __future__ import annotations

import torch

# No key index reaches it, so a row with this own-block start has no own-block term (plm/mask.py:14).
UNREACHABLE = 1 << 30


def round_layout(block_sizes: list[int], device: torch.device | str = "cpu"):
    """``(rel_positions, rel_aux, depth, own_start)`` per row of a round with ``len(block_sizes)`` verify rows,
    relative to its offset (plm/mask.py:42-65). Block d's row j sits at offset+d+j and reads the auxiliary cell of
    that position; verify rows are real tokens and read the masked sentinel (``rel_aux = -1``)."""
    n_hyp = len(block_sizes)
    rel_positions, rel_aux, depth, own_start = list(range(n_hyp)), [-1] * n_hyp, list(range(n_hyp)), \
        [UNREACHABLE] * n_hyp
    start = n_hyp
    for d, width in enumerate(block_sizes):
        for j in range(width):
            rel_positions.append(d + j)
            rel_aux.append(d + j)
            depth.append(d)
            own_start.append(start)
        start += width
    as_tensor = lambda v: torch.tensor(v, dtype=torch.int64, device=device)  # noqa: E731
    return as_tensor(rel_positions), as_tensor(rel_aux), as_tensor(depth), as_tensor(own_start)


def visible(depth: torch.Tensor, own_start: torch.Tensor, offset: int, q_idx: torch.Tensor,
            kv_idx: torch.Tensor) -> torch.Tensor:
    """The mask value for logical indices (RoundMaskView.__call__, plm/mask.py:23-29)."""
    row = q_idx - offset
    key = kv_idx - offset
    return (key <= depth[row]) | ((key >= own_start[row]) & (kv_idx <= q_idx))
