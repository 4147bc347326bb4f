"""The layer block's unit schedule (host code, run here without a GPU through plm_block_schedule).

The block's CTAs wait on counters that other CTAs' units advance, so the schedule must give every CTA its units in
phase order (o units, then norm rows, then gate_up tiles, then down units): a unit then only ever waits on units of
earlier phases, which every CTA of a fully resident grid reaches. These tests check that order, that every unit of
every phase is scheduled exactly once, and the balance of the down phase, for several model shapes and SM counts.
"""

from __future__ import annotations

import pytest

GATE, DOWN, O, NORM = 0, 1, 2, 3
PHASE = {O: 0, NORM: 1, GATE: 2, DOWN: 3}
MAX_ROWS = 128
STAGE_KB = 2  # k-blocks of 64 per ring stage


def _decode(code: int) -> tuple[int, int, int]:
    return (code >> 28) & 3, (code >> 12) & 0xFFFF, code & 0xFFF


SHAPES = {  # hidden, intermediate, q_size
    "plm-1.3b": (2048, 8192, 2048),
    "plm-3b": (2560, 10240, 2560),
    "gqa-1.3b": (2048, 5632, 2048),
    "small": (512, 2048, 512),
}


@pytest.mark.parametrize("sms", [148, 132, 160, 96])
@pytest.mark.parametrize("shape", list(SHAPES))
def test_schedule_covers_every_unit_once_in_phase_order(shape, sms):
    from plm import native

    hidden, inter, q_size = SHAPES[shape]
    lists = native.block_schedule(sms, hidden, inter, q_size)
    assert len(lists) == sms
    seen = {O: [], NORM: [], GATE: [], DOWN: []}
    for units in lists:
        phases = [PHASE[_decode(c)[0]] for c in units]
        assert phases == sorted(phases), "a CTA's units must come in phase order"
        for c in units:
            kind, tile, split = _decode(c)
            seen[kind].append((tile, split))
    o_tiles = down_tiles = -(-hidden // 128)
    o_splits = max(split for _, split in seen[O]) + 1
    down_splits = max(split for _, split in seen[DOWN]) + 1
    assert sorted(seen[O]) == [(t, s) for t in range(o_tiles) for s in range(o_splits)]
    assert o_tiles * o_splits <= max(sms, o_tiles)  # one o unit per CTA at most, so o does not queue
    assert sorted(seen[NORM]) == [(r, 0) for r in range(MAX_ROWS)]
    assert sorted(seen[GATE]) == [(t, 0) for t in range(inter // 64)]
    assert sorted(seen[DOWN]) == [(t, s) for t in range(down_tiles) for s in range(down_splits)]


@pytest.mark.parametrize("sms", [148, 132])
@pytest.mark.parametrize("shape", list(SHAPES))
def test_down_phase_is_balanced(shape, sms):
    """Down units are placed on the CTA with the fewest down k-blocks: no CTA carries more than one unit's worth of
    k-blocks above another."""
    from plm import native

    hidden, inter, q_size = SHAPES[shape]
    lists = native.block_schedule(sms, hidden, inter, q_size)
    pairs = inter // 64 // STAGE_KB
    splits = max(_decode(c)[2] for units in lists for c in units if _decode(c)[0] == DOWN) + 1

    def kb(split):
        return STAGE_KB * ((split + 1) * pairs // splits - split * pairs // splits)

    load = [sum(kb(_decode(c)[2]) for c in units if _decode(c)[0] == DOWN) for units in lists]
    assert max(load) - min(load) <= max(kb(s) for s in range(splits))


def test_unsupported_shapes_and_small_buffers_are_rejected():
    import ctypes

    from plm import native

    with pytest.raises(native.NativeError):
        native.block_schedule(148, 2000, 8192, 2048)  # hidden not a multiple of 128
    lib = native.library()
    n = ctypes.c_int32(0)
    offsets = (ctypes.c_int32 * 149)()
    units = (ctypes.c_int32 * 4)()
    assert lib.plm_block_schedule(148, 2048, 8192, 2048, units, 4, offsets, ctypes.byref(n)) != 0
    assert n.value > 4
