"""The PTP scheme's CPU restatement (oracle/ptp.py) against fixtures produced by the reference's own
LinearInterpolationAuxiliary and GatedLoraMethod (tests/golden/make_golden.py, section ptp)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ptp
from tests.golden import make_golden as mg

GOLDEN = np.load(Path(__file__).parent / "golden" / "ptp.npz")


def test_linear_interpolation_embed_matches_reference():
    seed, n, hidden, rows = mg.PTP_EMBED
    table, values = mg.ptp_embed_inputs(seed, n, hidden, rows)
    assert mg.checksum(table) + mg.checksum(values) == pytest.approx(float(GOLDEN["embed/checksum"]), rel=1e-12)
    got = ptp.linear_interpolation_embed(values.numpy(), table.numpy())
    np.testing.assert_array_equal(got, GOLDEN["embed/out"])
    # u = 0 is the first row, u = 0.5 the middle row of three: no blending error
    np.testing.assert_array_equal(got[0], table[0].numpy())
    np.testing.assert_array_equal(got[2], table[1].numpy())


@pytest.mark.parametrize("case", mg.PTP_DECODE)
def test_icdf_decode_matches_reference(case):
    seed, n, vocab, top_k = case
    logits, u = mg.ptp_decode_inputs(seed, n, vocab)
    assert mg.checksum(logits) + mg.checksum(u) == pytest.approx(float(GOLDEN[f"decode/{seed}/checksum"]), rel=1e-12)
    got = np.asarray([ptp.icdf_decode_row(logits[i].numpy(), float(u[i]), top_k) for i in range(n)])
    np.testing.assert_array_equal(got, GOLDEN[f"decode/{seed}/tokens"])


def test_icdf_bins_are_the_renormalised_top_k_in_token_order():
    logits = np.log(np.asarray([0.1, 0.4, 0.2, 0.3], dtype=np.float32))
    ids, edges = ptp.icdf_probabilities(logits, 3)
    np.testing.assert_array_equal(ids, [1, 2, 3])            # the top three, by token id
    np.testing.assert_allclose(edges, [4 / 9, 6 / 9, 1.0], rtol=1e-6)
    assert ptp.icdf_decode_row(logits, 0.0, 3) == 1
    assert ptp.icdf_decode_row(logits, 0.5, 3) == 2
    assert ptp.icdf_decode_row(logits, 0.99, 3) == 3


@pytest.mark.parametrize("case", mg.PTP_GATED)
def test_gated_projection_matches_reference(case):
    seed, dtype = case
    x, weight, lora_a, lora_bs = mg.ptp_gated_inputs(seed, dtype)
    tdtype = getattr(torch, dtype)
    rnd = lambda t: t.to(tdtype).to(torch.float32)  # noqa: E731
    mm = lambda a, b: a @ b  # noqa: E731
    f = lambda t: t.to(torch.float32)  # noqa: E731
    adapter = ptp.Adapter(f(lora_a), [f(b) for b in lora_bs])
    rows_from = mg.PTP_GATED_SHAPE["rows_from"]
    got = ptp.gated_projection(f(x), f(weight), adapter, rows_from, rnd, mm).numpy()
    ungated = ptp.gated_projection(f(x), f(weight), adapter, None, rnd, mm).numpy()
    ref, ref_ungated = GOLDEN[f"gated/{seed}/out"], GOLDEN[f"gated/{seed}/ungated"]
    # fp32: summation order only; bf16: at most one rounding step of the model dtype apart
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == "float32" else dict(rtol=1.6e-2, atol=1e-2)
    np.testing.assert_allclose(got, ref, **tol)
    np.testing.assert_allclose(ungated, ref_ungated, **tol)
    # rows before the first gated row are the base projection's, bit for bit
    np.testing.assert_array_equal(got[:rows_from], ungated[:rows_from])
    assert np.abs(got[rows_from:] - ungated[rows_from:]).max() > 0


def _ptp_round_oracles(k: int = 3):
    """Two PTP round oracles over the same small Llama: one with adapters on every projection, one without."""
    from oracle import model as omodel
    from oracle import rounds as orounds

    c = mg.LLAMA
    w = mg.llama_weights(c["seed"], c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"],
                         c["vocab"])
    shape = omodel.ModelShape(c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"],
                              c["vocab"], 64, max_pos=4096)
    g = torch.Generator().manual_seed(530)
    q_size, kv_size = c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    rank = 4
    shards = {"qkv": (q_size, kv_size, kv_size), "o": (c["hidden"],), "gate_up": (c["inter"], c["inter"]),
              "down": (c["hidden"],)}
    inputs = {"qkv": c["hidden"], "o": q_size, "gate_up": c["hidden"], "down": c["inter"]}
    adapters = [{name: ptp.Adapter(torch.randn(len(sh) * rank, inputs[name], generator=g) * 0.05,
                                   [torch.randn(width, rank, generator=g) * 0.05 for width in sh])
                 for name, sh in shards.items()} for _ in range(c["layers"])]
    scheme = ptp.PTPScheme(embedding=(torch.randn(3, c["hidden"], generator=g) * 0.02).numpy(), top_k=16)
    page, pages = 16, 16
    table = np.random.default_rng(1).permutation(pages)
    stream = torch.rand(orounds.AUX_STREAM_LENGTH, generator=g).numpy()
    make = lambda a: omodel.RoundOracle(  # noqa: E731
        omodel.OracleModel(shape, w, "float32", page, pages, table, ptp=scheme, adapters=a), None, k,
        aux_stream=stream.copy())
    return make(adapters), make(None), k


def test_ptp_round_oracle_gates_only_auxiliary_rows():
    """The reference keeps the text rows on the base weights (plm/gated_lora.py:1-7): the prefill, round 0's verify
    row and a steady round's k verify rows give the same logits with and without adapters, while the auxiliary rows
    differ."""
    from oracle import rounds as orounds

    gated, base, k = _ptp_round_oracles()
    prompt = np.random.default_rng(2).integers(0, mg.LLAMA["vocab"], 40)
    first_g, first_b = gated.prefill(prompt), base.prefill(prompt)
    np.testing.assert_array_equal(gated.last_logits, base.last_logits)
    assert first_g == first_b
    _, lg = gated.round0_forward()
    _, lb = base.round0_forward()
    np.testing.assert_array_equal(lg[:1], lb[:1])
    assert np.abs(lg[1:] - lb[1:]).max() > 0
    gated.commit_round0(lg[:1], orounds.argmax_first(lg[1:]))
    base.state = gated.state.copy()
    _, lg = gated.round_forward()
    _, lb = base.round_forward()
    np.testing.assert_array_equal(lg[:k], lb[:k])
    assert np.abs(lg[k:] - lb[k:]).max() > 0
    accepted = gated.commit_round(lg[:k], orounds.argmax_first(lg[k:]).reshape(k, k))
    assert 0 <= accepted <= k - 1


def test_ptp_verify_decode_reads_the_stream_at_base():
    """A steady round decodes verify row d at u = stream[base + d] (plm/decoder.py:262, 351-365): the token it
    commits after the nc accepted proposals is the inverse-CDF token of verify row nc."""
    from oracle import rounds as orounds

    gated, _, k = _ptp_round_oracles()
    gated.prefill(np.arange(1, 21))
    gated.round0()
    base_before = gated.state.base
    _, lg = gated.round_forward()
    nc = gated.commit_round(lg[:k], orounds.argmax_first(lg[k:]).reshape(k, k))
    expected = ptp.icdf_decode_row(lg[nc], float(gated.aux[base_before + nc]), 16)
    assert gated.state.out[base_before + nc] == expected
    assert gated.state.base == base_before + nc + 1
