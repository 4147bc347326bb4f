"""The PTP scheme's inverse-CDF verify decode on the GPU (plm_icdf_decode) against its CPU restatement
(oracle/ptp.py, itself pinned to the reference's LinearInterpolationAuxiliary in test_ptp_oracle.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ptp
from tests.golden import make_golden as mg

pytestmark = pytest.mark.gpu


def _run(ctx, logits: torch.Tensor, u: torch.Tensor, top_k: int):
    from plm import native

    n = logits.shape[0]
    tokens = torch.full((n,), -7, dtype=torch.int64, device="cuda")
    ids = torch.full((n, top_k), -7, dtype=torch.int32, device="cuda")
    edges = torch.full((n, top_k), -7.0, dtype=torch.float32, device="cuda")
    native.icdf_decode(ctx, logits.cuda().contiguous(), u.cuda().contiguous(), top_k, tokens, ids, edges)
    torch.cuda.synchronize()
    ctx.check()
    return tokens.cpu().numpy(), ids.cpu().numpy(), edges.cpu().numpy()


def _check_against_oracle(logits: torch.Tensor, u: torch.Tensor, top_k: int, got):
    tokens, ids, edges = got
    for r in range(logits.shape[0]):
        o_ids, o_edges = ptp.icdf_probabilities(logits[r].numpy(), top_k)
        np.testing.assert_array_equal(ids[r], o_ids)  # the same top_k set, in token-id order
        # float32 softmax terms and sums in another order: the edges agree to a few float32 steps
        np.testing.assert_allclose(edges[r], o_edges, rtol=0, atol=4e-6)
        assert edges[r][-1] == 1.0
        uu = float(u[r])
        if np.abs(o_edges - uu).min() > 1e-5:  # u not within rounding distance of an edge: the same bin
            assert tokens[r] == ptp.icdf_decode_row(logits[r].numpy(), uu, top_k)
        else:
            assert tokens[r] in o_ids


@pytest.mark.parametrize("case", mg.PTP_DECODE + ((513, 8, 50257, 128), (514, 3, 50257, 256)))
def test_icdf_decode_matches_oracle(ctx, case):
    seed, n, vocab, top_k = case
    logits, u = mg.ptp_decode_inputs(seed, n, vocab)
    _check_against_oracle(logits, u, top_k, _run(ctx, logits, u, top_k))


def test_icdf_decode_matches_reference_fixture(ctx):
    """The decoded tokens of the reference's own LinearInterpolationAuxiliary on the same inputs."""
    from pathlib import Path

    golden = np.load(Path(__file__).parent / "golden" / "ptp.npz")
    for seed, n, vocab, top_k in mg.PTP_DECODE:
        logits, u = mg.ptp_decode_inputs(seed, n, vocab)
        tokens, _, _ = _run(ctx, logits, u, top_k)
        np.testing.assert_array_equal(tokens, golden[f"decode/{seed}/tokens"])


def test_icdf_decode_ties_and_extremes(ctx):
    """Equal probabilities go to the lowest ids; u = 0 is the first chosen id, u just below 1 the last; a single
    dominant logit takes every bin below it."""
    vocab, top_k = 5000, 64
    logits = torch.zeros(4, vocab)
    logits[2, 4321] = 50.0
    logits[3, ::7] = 1.0  # 715 equal maxima, the top_k lowest of them chosen
    u = torch.tensor([0.0, 0.99999994, 0.5, 0.3])
    tokens, ids, edges = _run(ctx, logits, u, top_k)
    np.testing.assert_array_equal(ids[0], np.arange(top_k))
    np.testing.assert_allclose(edges[0], (np.arange(top_k) + 1) / top_k, atol=2e-6)
    assert tokens[0] == 0 and tokens[1] == top_k - 1
    assert tokens[2] == 4321
    np.testing.assert_array_equal(ids[3], np.arange(top_k) * 7)
    _check_against_oracle(logits, u, top_k, (tokens, ids, edges))


def test_icdf_decode_rejects_bad_shapes(ctx):
    from plm import native

    logits = torch.zeros(2, 300, device="cuda")
    u = torch.zeros(2, device="cuda")
    tokens = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(native.NativeError):
        native.icdf_decode(ctx, logits, u, 257, tokens)
    with pytest.raises(native.NativeError):
        native.icdf_decode(ctx, logits, u, 301, tokens)
    with pytest.raises(native.NativeError):
        native.icdf_decode(ctx, torch.zeros(1, 60000, device="cuda"), u, 16, tokens)
