"""Restatement of the round's layout, mask and loop-carried bookkeeping (test infrastructure).

Follows plm/mask.py (round_layout, RoundMaskView) and the RoundDecoder pieces of plm/decoder.py that are integer
work: the prologue's ids / auxiliary values / positions / slots (331-349), the steady epilogue (351-365), round 0
(275-310) and the first token after the prefill (384, with round 0's state reset 279-284). All arrays are numpy
int64 on the CPU.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

UNREACHABLE = 1 << 30  # plm/mask.py:14
AUX_STREAM_LENGTH = 8192  # plm/decoder.py:28
SEQUENCE_CAPACITY = 1 << 17  # plm/decoder.py:86


def round_layout(block_sizes: list[int]):
    """(rel_positions, rel_aux, depth, own_start) per row, relative to the round offset (plm/mask.py:42-65)."""
    n_hyp = len(block_sizes)
    rel_positions, rel_aux, depth, own_start = [], [], [], []
    for d in range(n_hyp):  # verify rows: real tokens, causal among themselves
        rel_positions.append(d)
        rel_aux.append(-1)
        depth.append(d)
        own_start.append(UNREACHABLE)
    start = n_hyp
    for d, width in enumerate(block_sizes):  # block d row j: sits at offset+d+j, reads that position's auxiliary
        for j in range(width):
            rel_positions.append(d + j)
            rel_aux.append(d + j)
            depth.append(d)
            own_start.append(start)
        start += width
    as_array = lambda v: np.asarray(v, dtype=np.int64)  # noqa: E731
    return as_array(rel_positions), as_array(rel_aux), as_array(depth), as_array(own_start)


def steady_layout(k: int):
    return round_layout([k] * k)


def round0_layout(k: int):
    return round_layout([k + k * k - 1])


def chunk_layout(width: int):
    """A causal prefill chunk: depth = row, no own block (plm/decoder.py:372-373)."""
    rows = np.arange(width, dtype=np.int64)
    return rows, np.full(width, -1, dtype=np.int64), rows, np.full(width, UNREACHABLE, dtype=np.int64)


def visible(depth: np.ndarray, own_start: np.ndarray, offset: int, n_keys: int) -> np.ndarray:
    """[rows, n_keys] mask: key kv visible to row r iff kv-off <= depth[r] or (kv-off >= own_start[r] and kv <= q),
    with q = offset + r, and kv < offset + rows (plm/mask.py:23-29 under the backend's sequence length)."""
    rows = depth.size
    q = offset + np.arange(rows, dtype=np.int64)[:, None]
    kv = np.arange(n_keys, dtype=np.int64)[None, :]
    key = kv - offset
    prefix = key <= depth[:, None]
    own = (key >= own_start[:, None]) & (kv <= q)
    return (prefix | own) & (kv < offset + rows)


@dataclass
class RoundState:
    """The RoundDecoder's loop-carried device state (plm/decoder.py:119-146)."""
    k: int
    capacity: int
    offset: int = 0
    base: int = 0
    anchor: int = 0
    pending: np.ndarray = None
    out: np.ndarray = None
    round_sequence: list = field(default_factory=list)

    def __post_init__(self):
        if self.pending is None:
            self.pending = np.zeros(self.k - 1, dtype=np.int64)
        if self.out is None:
            self.out = np.full(self.capacity, -1, dtype=np.int64)

    def copy(self) -> "RoundState":
        return RoundState(self.k, self.capacity, self.offset, self.base, self.anchor, self.pending.copy(),
                          self.out.copy(), list(self.round_sequence))


def prologue(state: RoundState, layout, vocab: int, sentinel: int, aux_buf: np.ndarray):
    """ids, auxiliary values, rotary positions and logical KV slots of a steady round (plm/decoder.py:331-349).

    The reference's slot_mapping adds the null page (``+ BS``, decoder.py:347); here slots are logical KV indices
    (offset + row) and the block table maps them to pages."""
    rel_positions, rel_aux, _, _ = layout
    k = state.k
    width = rel_positions.size
    ids = np.full(width, vocab, dtype=np.int64)
    ids[0] = state.anchor
    ids[1:k] = state.pending
    aux_index = state.base + rel_aux
    aux_values = np.where(rel_aux < 0, sentinel, aux_buf[np.maximum(aux_index, 0)])
    positions = rel_positions + state.offset
    slots = state.offset + np.arange(width, dtype=np.int64)
    return ids, aux_values.astype(aux_buf.dtype), positions, slots


def round0_prologue(state: RoundState, layout, vocab: int, sentinel: int, aux_buf: np.ndarray):
    """Round 0's inputs (plm/decoder.py:288-296): the anchor, then W-1 proposal rows."""
    rel_positions, rel_aux, _, _ = layout
    width = rel_positions.size
    ids = np.full(width, vocab, dtype=np.int64)
    ids[0] = state.anchor
    aux_index = state.base + rel_aux
    aux_values = np.where(rel_aux < 0, sentinel, aux_buf[np.maximum(aux_index, 0)])
    return ids, aux_values.astype(aux_buf.dtype), rel_positions + state.offset, state.offset + np.arange(width)


def epilogue(state: RoundState, verify: np.ndarray, accepted_rule: np.ndarray, proposal_argmax: np.ndarray) -> int:
    """Steady-round acceptance and commit (plm/decoder.py:351-365). ``proposal_argmax`` is [k, k]: the argmax token
    of every proposal row, block-major. Mutates ``state``; returns the accepted count."""
    k = state.k
    accepted = (verify[: k - 1] == state.pending) | accepted_rule[: k - 1].astype(bool)
    num_correct = int(np.cumprod(accepted.astype(np.int64)).sum())
    confirmed_head = np.concatenate([state.pending, verify[-1:]])
    picked = int(verify[min(num_correct, k - 1)])
    for j in range(k):
        slot = state.base + j
        if j < num_correct:
            state.out[slot] = confirmed_head[j]
        elif j == num_correct:
            state.out[slot] = picked
    state.round_sequence.append(num_correct)
    state.pending = proposal_argmax.reshape(k, k)[num_correct, 1:k].astype(np.int64).copy()
    state.anchor = picked
    state.base += num_correct + 1
    state.offset += num_correct + 1
    return num_correct


def round0_epilogue(state: RoundState, verify0: int, hypotheses: np.ndarray) -> None:
    """Round 0's commit (plm/decoder.py:299-310): nothing accepted, ``hypotheses`` = argmax of rows 1..W-1."""
    k = state.k
    state.out[state.base] = verify0
    state.pending = np.asarray(hypotheses[1:k], dtype=np.int64).copy()
    state.anchor = int(verify0)
    state.base += 1
    state.offset += 1


def first_token(state: RoundState, first: int, prompt_len: int) -> None:
    """The prefill's decoded token and round 0's state reset (plm/decoder.py:279-284, 384)."""
    state.out[:] = -1
    state.out[0] = first
    state.base = 1
    state.anchor = int(first)
    state.pending = np.zeros(state.k - 1, dtype=np.int64)
    state.offset = prompt_len


def argmax_first(values: np.ndarray) -> np.ndarray:
    """Row argmax with the first index on ties (torch.argmax's documented choice)."""
    return np.argmax(values, axis=-1)


def commit_rows(cache: np.ndarray, scratch: np.ndarray, block_table: np.ndarray, page_size: int, first: int,
                count: int) -> None:
    """The KV commit of a round, in place: rows 0 .. count-1 of the round's K/V (``scratch``
    [layers][2][rows][kv_heads][head_dim]) go to logical KV indices first .. first+count-1 of the paged ``cache``
    [layers][2][pages][kv_heads][page_size][head_dim] through the block table. This is the reference's implicit
    commit made explicit: plm/decoder.py:351-365 advances the offset over the verify rows 0 .. nc that the forward
    already wrote in place, and eagle3/tree.py:263-279 moves accepted rows into their final slots the same way
    (kv[dst // BS, :, dst % BS, :] = ...)."""
    for j in range(count):
        logical = first + j
        page = int(block_table[logical // page_size])
        cache[:, :, page, :, logical % page_size, :] = scratch[:, :, j, :, :]
