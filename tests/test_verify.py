"""plm_verify_decode against the oracle, bit for bit, on identical fp32 logits and cost table.

Checked per row: softmax statistics, shortlist tokens and quotas, fitted factors, the decoded token, the relaxed
acceptance verdicts, and the round bookkeeping the last CTA performs (steady round, round 0, first token).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rounds as orounds
from oracle import voronoi as ov

pytestmark = pytest.mark.gpu


def _bits(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).view(np.int32)


def _logits(kind: str, n: int, vocab: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(n, vocab, generator=g, device="cuda") * 2.0
    if kind == "bf16":
        x = x.bfloat16().float()
    elif kind == "flat":
        x = torch.zeros_like(x)
    elif kind == "coarse":  # many equal values at the top-128 boundary
        x = torch.round(x * 4) / 4
    elif kind == "peaked":
        x = x.bfloat16().float()
        x[:, 17] = 60.0
    return x.contiguous()


def _table(vocab: int, aux: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(vocab, aux, generator=g, device="cuda") * 0.3).bfloat16().contiguous()


def run_verify(ctx, logits, table, cells, *, pending=None, rule=0, threshold=-1.0, top_m=128, shortlist=8,
               rounds=2, sweeps=12, book=None, aux_base=None, aux_buf=None):
    from plm import native

    n, vocab = logits.shape
    aux = table.shape[1]
    if aux_buf is None:
        aux_buf = torch.tensor(cells, dtype=torch.int64, device="cuda")
    out = {
        "verify": torch.full((n,), -7, dtype=torch.int64, device="cuda"),
        "flags": torch.full((n,), -7, dtype=torch.int32, device="cuda"),
        "tokens": torch.zeros(n, top_m, dtype=torch.int32, device="cuda"),
        "counts": torch.zeros(n, top_m, dtype=torch.int32, device="cuda"),
        "bias": torch.zeros(n, top_m, dtype=torch.float32, device="cuda"),
        "stats": torch.zeros(n, 4, dtype=torch.float32, device="cuda"),
        "sigma": torch.zeros(n, dtype=torch.int32, device="cuda"),
    }
    desc = native.VerifyDesc(
        dtype=native.PLM_BF16, logits=logits.data_ptr(), n_rows=n, vocab=vocab, logits_stride=vocab,
        table=table.data_ptr(), aux=aux, aux_buf=aux_buf.data_ptr(), aux_len=aux_buf.numel(),
        aux_base=None if aux_base is None else aux_base.data_ptr(), aux_row_offset=0,
        pending=None if pending is None else pending.data_ptr(), n_accept=0 if pending is None else pending.numel(),
        rule=rule, threshold=threshold, top_m=top_m, shortlist=shortlist, rounds=rounds, sweeps=sweeps,
        epsilon=0.15, refocus=0.35, endpoint=0.0087, verify=out["verify"].data_ptr(), flags=out["flags"].data_ptr(),
        dbg_tokens=out["tokens"].data_ptr(), dbg_counts=out["counts"].data_ptr(), dbg_bias=out["bias"].data_ptr(),
        dbg_stats=out["stats"].data_ptr(), dbg_sigma=out["sigma"].data_ptr(),
        book=book if book is not None else native.Bookkeeping(mode=native.BOOK_NONE))
    native.verify_decode(ctx, desc)
    ctx.check()
    return {key: value.cpu().numpy() for key, value in out.items()}


def _check_rows(gpu, logits_np, table_np, cells, config):
    for r in range(logits_np.shape[0]):
        ref = ov.decode_row(logits_np[r], table_np, cells[r], "bfloat16", config)
        stats = gpu["stats"][r]
        assert _bits(stats[0]) == _bits(ref.maximum), f"row {r}: max"
        assert _bits(stats[1]) == _bits(ref.total), f"row {r}: sum of exp"
        assert _bits(stats[2]) == _bits(ref.normaliser), f"row {r}: normaliser"
        assert _bits(stats[3]) == _bits(ref.unit), f"row {r}: unit"
        np.testing.assert_array_equal(gpu["tokens"][r], ref.tokens, err_msg=f"row {r}: shortlist")
        np.testing.assert_array_equal(gpu["counts"][r], ref.counts, err_msg=f"row {r}: quota")
        assert gpu["counts"][r].sum() == table_np.shape[1]
        np.testing.assert_array_equal(_bits(gpu["bias"][r]), _bits(ref.bias), err_msg=f"row {r}: fitted factors")
        assert gpu["sigma"][r] == ref.sigma, f"row {r}: sigma"
        assert gpu["verify"][r] == ref.token, f"row {r}: token"


@pytest.mark.parametrize("kind", ["bf16", "fp32", "coarse", "flat", "peaked"])
def test_verify_decode_bit_exact(ctx, kind):
    vocab, aux, n = 50257, 1024, 3
    logits = _logits(kind, n, vocab, seed=21)
    table = _table(vocab, aux, seed=22)
    cells = [5, 700, 1023]
    gpu = run_verify(ctx, logits, table, cells)
    _check_rows(gpu, logits.cpu().numpy(), table.float().cpu().numpy(), cells, ov.VoronoiConfig())


@pytest.mark.parametrize("vocab,aux,top_m,shortlist", [(3000, 256, 128, 8), (5000, 4096, 128, 8), (2048, 512, 64, 4),
                                                       (700, 32, 32, 2)])
def test_verify_decode_shapes(ctx, vocab, aux, top_m, shortlist):
    n = 2
    logits = _logits("bf16", n, vocab, seed=23)
    table = _table(vocab, aux, seed=24)
    cells = [0, aux - 1]
    config = ov.VoronoiConfig(top_m=top_m, shortlist=shortlist)
    gpu = run_verify(ctx, logits, table, cells, top_m=top_m, shortlist=shortlist)
    _check_rows(gpu, logits.cpu().numpy(), table.float().cpu().numpy(), cells, config)


@pytest.mark.parametrize("rule,threshold", [(0, 0.94), (0, 0.5), (1, 2e-3), (1, 1e-4), (0, -1.0)])
def test_acceptance_rules_bit_exact(ctx, rule, threshold):
    from plm import native

    vocab, aux, n = 50257, 256, 7
    logits = _logits("bf16", n, vocab, seed=25)
    # make the proposals land at a range of ranks so some pass and some fail
    order = torch.argsort(logits, dim=-1, descending=True)
    ranks = torch.tensor([0, 1, 3, 10, 50, 400, 20000], device="cuda")
    pending = order[torch.arange(n, device="cuda"), ranks].contiguous()
    table = _table(vocab, aux, seed=26)
    gpu = run_verify(ctx, logits, table, [1] * n, pending=pending, rule=rule, threshold=threshold)
    logits_np, pend = logits.cpu().numpy(), pending.cpu().numpy()
    for r in range(n):
        if rule == native.RULE_FLOOR:
            expect = ov.floor_accepts(logits_np[r], int(pend[r]), threshold)
        else:
            expect = ov.nucleus_accepts(logits_np[r], int(pend[r]), threshold)
        assert bool(gpu["flags"][r]) == expect, f"row {r} rank {int(ranks[r])}"
    if threshold <= 0:
        assert not gpu["flags"].any()


def _partials(tiles: int, rows: int, vocab: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    val = torch.randint(0, 6, (tiles, rows), generator=g, device="cuda").float()  # many ties
    idx = torch.arange(tiles, device="cuda")[:, None] * 128 + torch.randint(0, 128, (tiles, rows), generator=g,
                                                                             device="cuda")
    return val.contiguous(), idx.clamp(max=vocab - 1).to(torch.int32).contiguous()


def _expected_argmax(val: np.ndarray, idx: np.ndarray) -> np.ndarray:
    out = []
    for r in range(val.shape[1]):
        top = val[:, r].max()
        out.append(idx[val[:, r] == top, r].min())
    return np.asarray(out, dtype=np.int64)


@pytest.mark.parametrize("nc_target,rule,threshold", [(0, 0, -1.0), (3, 0, -1.0), (6, 0, -1.0), (2, 0, 0.94),
                                                      (1, 1, 2e-3)])
def test_steady_bookkeeping(ctx, nc_target, rule, threshold):
    """Acceptance + commit of a steady round against the restatement of plm/decoder.py:351-365."""
    from plm import native

    k, vocab, aux = 7, 50257, 256
    width = k + k * k
    logits = _logits("bf16", k, vocab, seed=27 + nc_target)
    table = _table(vocab, aux, seed=28)
    aux_stream = torch.randint(0, aux, (8192,), device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    base0, offset0, cap = 40, 1100, 4096
    # decode once without bookkeeping to learn the verify tokens, then plant proposals that match the first
    # nc_target of them
    probe = run_verify(ctx, logits, table, None, aux_base=torch.tensor([base0], device="cuda"), aux_buf=aux_stream)
    verify = probe["verify"]
    pending = torch.tensor([(int(verify[j]) if j < nc_target else (int(verify[j]) + 1) % vocab) for j in range(k - 1)],
                           dtype=torch.int64, device="cuda")
    tiles = native.gemm_tiles(native.EPI_LOGITS, vocab)
    best_val, best_idx = _partials(tiles, width, vocab, seed=29)
    out = torch.full((cap,), -1, dtype=torch.int64, device="cuda")
    out[:base0] = torch.arange(base0, device="cuda")
    state = {name: torch.tensor([v], dtype=torch.int64, device="cuda")
             for name, v in (("base", base0), ("offset", offset0), ("anchor", 99), ("step", 5))}
    round_sequence = torch.zeros(64, dtype=torch.int64, device="cuda")
    pend_dev = pending.clone()
    book = native.Bookkeeping(mode=native.BOOK_STEADY, k=k, best_val=best_val.data_ptr(), best_idx=best_idx.data_ptr(),
                              n_tiles=tiles, rows=width, out=out.data_ptr(), out_cap=cap,
                              base=state["base"].data_ptr(), offset=state["offset"].data_ptr(),
                              anchor=state["anchor"].data_ptr(), pending=pend_dev.data_ptr(),
                              round_sequence=round_sequence.data_ptr(), seq_cap=64,
                              sequence_step=state["step"].data_ptr())
    gpu = run_verify(ctx, logits, table, None, pending=pend_dev, rule=rule, threshold=threshold, book=book,
                     aux_base=state["base"], aux_buf=aux_stream)
    # oracle
    ref = orounds.RoundState(k, cap, offset=offset0, base=base0, anchor=99, pending=pending.cpu().numpy().copy(),
                             out=np.concatenate([np.arange(base0), np.full(cap - base0, -1)]).astype(np.int64))
    ref.round_sequence = [0] * 5
    logits_np = logits.cpu().numpy()
    rule_flags = np.zeros(k, dtype=bool)
    for r in range(k - 1):
        if rule == native.RULE_FLOOR:
            rule_flags[r] = ov.floor_accepts(logits_np[r], int(pending[r]), threshold)
        else:
            rule_flags[r] = ov.nucleus_accepts(logits_np[r], int(pending[r]), threshold)
    argmax_rows = _expected_argmax(best_val.cpu().numpy(), best_idx.cpu().numpy())
    nc = orounds.epilogue(ref, gpu["verify"], rule_flags, argmax_rows[k:])
    if rule == 0 and threshold <= 0:
        assert nc == nc_target
    np.testing.assert_array_equal(gpu["verify"], verify)
    np.testing.assert_array_equal(out.cpu().numpy(), ref.out)
    assert int(state["base"]) == ref.base and int(state["offset"]) == ref.offset
    assert int(state["anchor"]) == ref.anchor and int(state["step"]) == 6
    assert int(round_sequence[5]) == nc
    np.testing.assert_array_equal(pend_dev.cpu().numpy(), ref.pending)


def test_round0_and_first_token_bookkeeping(ctx):
    from plm import native

    k, vocab, aux, cap = 7, 50257, 256, 2048
    width = k + k * k
    logits = _logits("bf16", 1, vocab, seed=31)
    table = _table(vocab, aux, seed=32)
    aux_stream = torch.randint(0, aux, (8192,), device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    out = torch.full((cap,), 5, dtype=torch.int64, device="cuda")
    state = {name: torch.tensor([v], dtype=torch.int64, device="cuda")
             for name, v in (("base", 17), ("offset", 3), ("anchor", 1), ("step", 0))}
    pend = torch.full((k - 1,), 9, dtype=torch.int64, device="cuda")
    tiles = native.gemm_tiles(native.EPI_LOGITS, vocab)
    best_val, best_idx = _partials(tiles, width, vocab, seed=33)

    def book(mode):
        return native.Bookkeeping(mode=mode, k=k, best_val=best_val.data_ptr(), best_idx=best_idx.data_ptr(),
                                  n_tiles=tiles, rows=width, out=out.data_ptr(), out_cap=cap,
                                  base=state["base"].data_ptr(), offset=state["offset"].data_ptr(),
                                  anchor=state["anchor"].data_ptr(), pending=pend.data_ptr(), prompt_len=256)

    # first token after the prefill: aux cell 0 of the stream, absolute
    first = run_verify(ctx, logits, table, None, aux_buf=aux_stream, book=book(native.BOOK_FIRST_TOKEN))
    ref = orounds.RoundState(k, cap)
    token = ov.decode_row(logits.cpu().numpy()[0], table.float().cpu().numpy(), int(aux_stream[0]), "bfloat16").token
    assert int(first["verify"][0]) == token
    orounds.first_token(ref, token, 256)
    np.testing.assert_array_equal(out.cpu().numpy(), ref.out)
    assert (int(state["base"]), int(state["offset"]), int(state["anchor"])) == (ref.base, ref.offset, ref.anchor)
    assert (pend.cpu().numpy() == 0).all()

    # round 0: one verify row reading aux_stream[base]
    r0 = run_verify(ctx, logits, table, None, aux_base=state["base"], aux_buf=aux_stream, book=book(native.BOOK_ROUND0))
    token0 = ov.decode_row(logits.cpu().numpy()[0], table.float().cpu().numpy(), int(aux_stream[1]), "bfloat16").token
    assert int(r0["verify"][0]) == token0
    hyp = np.concatenate([[0], _expected_argmax(best_val.cpu().numpy(), best_idx.cpu().numpy())[1:]])
    orounds.round0_epilogue(ref, token0, hyp[1:])
    np.testing.assert_array_equal(out.cpu().numpy(), ref.out)
    assert (int(state["base"]), int(state["offset"]), int(state["anchor"])) == (ref.base, ref.offset, ref.anchor)
    np.testing.assert_array_equal(pend.cpu().numpy(), ref.pending)
