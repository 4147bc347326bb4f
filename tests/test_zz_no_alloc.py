"""plm_verify_decode_static, called through the C ABI, against plm_verify_decode on the same inputs.

The static entry point allocates nothing: its scratch is a file-scope device array. Each case makes two calls in a
row (the second reuses the scratch the first left behind: the arrival counter must be back at zero) and compares
every output bit for bit with the context entry point. The file is named to be collected last, so that it also runs
after every other GPU test has used the device; it passes alone as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

K, VOCAB, AUX = 7, 50257, 256


def _inputs(seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = (torch.randn(K, VOCAB, generator=g, device="cuda") * 2.0).bfloat16().float().contiguous()
    table = (torch.randn(VOCAB, AUX, generator=g, device="cuda") * 0.3).bfloat16().contiguous()
    aux_buf = torch.randint(0, AUX, (4096,), generator=g, device="cuda")
    return logits, table, aux_buf


def _desc(logits, table, aux_buf, *, verify=None, flags=None, pending=None, aux_base=None, book=None,
          rule=0, threshold=-1.0):
    from plm import native

    return native.VerifyDesc(
        dtype=native.PLM_BF16, logits=logits.data_ptr(), n_rows=logits.shape[0], vocab=VOCAB, logits_stride=VOCAB,
        table=table.data_ptr(), aux=AUX, aux_buf=aux_buf.data_ptr(), aux_len=aux_buf.numel(),
        aux_base=None if aux_base is None else aux_base.data_ptr(), aux_row_offset=0,
        pending=None if pending is None else pending.data_ptr(), n_accept=0 if pending is None else pending.numel(),
        rule=rule, threshold=threshold, top_m=128, shortlist=8, rounds=2, sweeps=12, epsilon=0.15, refocus=0.35,
        endpoint=0.0087, verify=None if verify is None else verify.data_ptr(),
        flags=None if flags is None else flags.data_ptr(),
        book=book if book is not None else native.Bookkeeping(mode=native.BOOK_NONE))


def _call_static(desc, device_error) -> int:
    from plm import native

    stream = ctypes.c_void_p(native.stream_handle())
    return native.library().plm_verify_decode_static(ctypes.byref(desc), ctypes.c_void_p(device_error.data_ptr()),
                                                     stream)


def test_decode_matches_context_entry_point(ctx):
    from plm import native

    device_error = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed in (11, 12):  # two calls in a row
        logits, table, aux_buf = _inputs(seed)
        pending = torch.randint(0, VOCAB, (K - 1,), device="cuda")
        want_v = torch.full((K,), -7, dtype=torch.int64, device="cuda")
        want_f = torch.full((K,), -7, dtype=torch.int32, device="cuda")
        native.verify_decode(ctx, _desc(logits, table, aux_buf, verify=want_v, flags=want_f, pending=pending,
                                        threshold=0.94))
        ctx.check()
        got_v = torch.full((K,), -9, dtype=torch.int64, device="cuda")
        got_f = torch.full((K,), -9, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        st = _call_static(_desc(logits, table, aux_buf, verify=got_v, flags=got_f, pending=pending, threshold=0.94),
                          device_error)
        assert st == native.PLM_OK, native.last_error()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before  # nothing was allocated on the device
        np.testing.assert_array_equal(got_v.cpu().numpy(), want_v.cpu().numpy())
        np.testing.assert_array_equal(got_f.cpu().numpy(), want_f.cpu().numpy())
    assert int(device_error) == 0


def _steady_state(seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    width = K + K * K
    tiles = 8
    best_val = torch.randint(0, 6, (tiles, width), generator=g, device="cuda").float().contiguous()
    best_idx = (torch.arange(tiles, device="cuda")[:, None] * 128
                + torch.randint(0, 128, (tiles, width), generator=g, device="cuda")).to(torch.int32).contiguous()
    cap, base0 = 1024, 40
    out = torch.full((cap,), -1, dtype=torch.int64, device="cuda")
    out[:base0] = torch.arange(base0, device="cuda")
    return {
        "best_val": best_val, "best_idx": best_idx, "tiles": tiles, "width": width, "cap": cap, "out": out,
        "base": torch.tensor([base0], dtype=torch.int64, device="cuda"),
        "offset": torch.tensor([700], dtype=torch.int64, device="cuda"),
        "anchor": torch.tensor([99], dtype=torch.int64, device="cuda"),
        "step": torch.tensor([0], dtype=torch.int64, device="cuda"),
        "pending": torch.randint(0, VOCAB, (K - 1,), generator=g, device="cuda"),
        "round_sequence": torch.zeros(16, dtype=torch.int64, device="cuda"),
    }


def _book(st):
    from plm import native

    return native.Bookkeeping(mode=native.BOOK_STEADY, k=K, best_val=st["best_val"].data_ptr(),
                              best_idx=st["best_idx"].data_ptr(), n_tiles=st["tiles"], rows=st["width"],
                              out=st["out"].data_ptr(), out_cap=st["cap"], base=st["base"].data_ptr(),
                              offset=st["offset"].data_ptr(), anchor=st["anchor"].data_ptr(),
                              pending=st["pending"].data_ptr(), round_sequence=st["round_sequence"].data_ptr(),
                              seq_cap=16, sequence_step=st["step"].data_ptr())


def test_steady_round_bookkeeping_matches_context_entry_point(ctx):
    """Two steady rounds in a row; the static calls keep the decoded tokens and verdicts in the scratch's row
    slots (verify and flags NULL) and use its arrival counter."""
    from plm import native

    ref, mine = _steady_state(5), _steady_state(5)
    device_error = torch.zeros(1, dtype=torch.int32, device="cuda")
    for seed in (21, 22):
        logits, table, aux_buf = _inputs(seed)
        verify = torch.zeros(K, dtype=torch.int64, device="cuda")
        flags = torch.zeros(K, dtype=torch.int32, device="cuda")
        native.verify_decode(ctx, _desc(logits, table, aux_buf, verify=verify, flags=flags, pending=ref["pending"],
                                        aux_base=ref["base"], book=_book(ref), rule=native.RULE_FLOOR,
                                        threshold=2e-3))
        ctx.check()
        st = _call_static(_desc(logits, table, aux_buf, pending=mine["pending"], aux_base=mine["base"],
                                book=_book(mine), rule=native.RULE_FLOOR, threshold=2e-3), device_error)
        assert st == native.PLM_OK, native.last_error()
        torch.cuda.synchronize()
        for name in ("out", "base", "offset", "anchor", "step", "pending", "round_sequence"):
            np.testing.assert_array_equal(mine[name].cpu().numpy(), ref[name].cpu().numpy(), err_msg=name)
    assert int(device_error) == 0
    assert int(mine["step"]) == 2


def test_rows_beyond_the_scratch_are_rejected():
    from plm import native

    logits = torch.zeros(33, VOCAB, device="cuda")
    table = torch.zeros(VOCAB, AUX, dtype=torch.bfloat16, device="cuda")
    aux_buf = torch.zeros(64, dtype=torch.int64, device="cuda")
    device_error = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _call_static(_desc(logits, table, aux_buf), device_error)
    assert native.STATUS_NAMES.get(st) == "PLM_ERR_INVALID"
    assert "static scratch" in native.last_error()
