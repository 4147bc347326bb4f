"""The PTP round (the reference's gated-LoRA distilled model, plm/gated_lora.py:35-90 with the linear-interpolation
scheme of plm/auxiliary.py:78-113) on the GPU against the CPU oracle's PTP model (oracle/ptp.py).

Teacher-forced, stage by stage as for the PLM round: prefill, round 0, steady rounds, both sides on the same state.
The GPU runs its base projections, the adapters' two GEMMs per shard on the gated rows (row 1 on in round 0, row k
on in a steady round, none in the prefill), the interpolated embeddings of the auxiliary rows, and the inverse-CDF
verify decode at the request's uniforms. Logits agree within 2e-2; given the GPU's logits, the decoded tokens,
acceptance and bookkeeping match the oracle bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import model as omodel
from oracle import ptp as optp
from oracle import voronoi as ov
from tests.test_round import _argmax_partials, _assert_state, _close

pytestmark = pytest.mark.gpu


def _ptp_pair(k: int, seed: int, rule: str, threshold, projections, page: int = 16):
    from plm.decoder import AUX_STREAM_LENGTH, RoundDecoder
    from plm.model import PLMWeights, shape_config

    cfg = shape_config("plm-tiny")
    weights = PLMWeights.random(cfg, seed=seed).with_ptp(rank=64, num_embeddings=3, top_k=128, seed=seed + 1,
                                                          projections=projections)
    max_model_len = 512
    probe_pages = -(-(max_model_len + 2 * (k + k * k) + page) // page)
    num_pages = probe_pages + 8
    table = np.random.default_rng(seed).permutation(num_pages)[:probe_pages].astype(np.int32)
    page_bytes = cfg.num_layers * 2 * cfg.num_kv_heads * page * cfg.head_dim * 2
    decoder = RoundDecoder(weights, k, rule, threshold, block_size=page, kv_cache_bytes=num_pages * page_bytes,
                           max_model_len=max_model_len, block_table=table.tolist())
    shape = omodel.ModelShape(cfg.num_layers, cfg.hidden, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                              cfg.intermediate, cfg.vocab, cfg.aux_vocab, cfg.num_aux_tokens, cfg.rms_eps,
                              cfg.rope_theta, decoder.cos_sin.shape[0])
    named = {key: ([t.cpu() for t in v] if isinstance(v, list) else v.cpu()) for key, v in weights.named().items()}
    adapters = []
    for layer, per in enumerate(weights.adapters):
        entry = {}
        for name, (lora_a, lora_b) in per.items():
            widths = weights.adapter_shards(layer, name)
            entry[name] = optp.Adapter(lora_a.float().cpu(), list(lora_b.float().cpu().split(widths)))
        adapters.append(entry)
    scheme = optp.PTPScheme(embedding=weights.ptp_embedding.cpu().numpy(), top_k=weights.ptp_top_k)
    model = omodel.OracleModel(shape, named, "bfloat16", page, num_pages, table, cos_sin=decoder.cos_sin.cpu(),
                               ptp=scheme, adapters=adapters)
    decoder._fill_aux(seed)
    uniforms = torch.rand(AUX_STREAM_LENGTH, dtype=torch.float32, device="cuda",
                          generator=torch.Generator(device="cuda").manual_seed(seed)).cpu().numpy()
    oracle = omodel.RoundOracle(model, None, k, rule, threshold, ov.VoronoiConfig(cfg.top_m, cfg.shortlist,
                                                                                  cfg.rounds, cfg.sweeps),
                                capacity=decoder.out.numel(), aux_stream=uniforms)
    return decoder, oracle, cfg


@pytest.mark.parametrize("k,rule,threshold,projections", [
    (7, "nucleus", None, ("qkv", "o", "gate_up", "down")),
    (4, "nucleus", 0.94, ("qkv", "o", "gate_up", "down")),
    (6, "floor", 2e-3, ("qkv", "down")),
])
def test_ptp_round_parity_teacher_forced(k, rule, threshold, projections):
    decoder, oracle, cfg = _ptp_pair(k, seed=5, rule=rule, threshold=threshold, projections=projections)
    report = {}
    prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(8))
    W = decoder.width

    decoder.handle.load_prompt(prompt.pin_memory())
    decoder.handle.prefill()
    decoder.check()
    _, logits_o = oracle.prefill_forward(prompt.numpy())
    gpu_logits = decoder.verify_logits[0].cpu().numpy()
    _close("prefill logits", gpu_logits, logits_o[0], report)
    oracle.commit_first(gpu_logits, prompt.numel())
    _assert_state(decoder, oracle.state)

    decoder.handle.round0()
    decoder.check()
    _, logits_o = oracle.round0_forward()
    gpu_logits = decoder.verify_logits[0].cpu().numpy()
    _close("round0 logits", gpu_logits, logits_o[0], report)
    oracle.commit_round0(gpu_logits[None], _argmax_partials(decoder, W)[1:])
    _assert_state(decoder, oracle.state)

    seq0 = int(decoder.sequence_step[0])
    for _ in range(5):
        decoder.handle.round()
        decoder.check()
        _, logits_o = oracle.round_forward()
        gpu_logits = decoder.verify_logits.cpu().numpy()
        _close("round logits", gpu_logits, logits_o[:k], report)
        oracle.commit_round(gpu_logits, _argmax_partials(decoder, W)[k:])
        _assert_state(decoder, oracle.state)
    assert decoder.round_sequence[seq0:int(decoder.sequence_step[0])].cpu().tolist() == oracle.state.round_sequence
    decoder.close()


def test_ptp_adapters_change_only_the_gated_rows():
    """The adapters act on a round's auxiliary rows only (plm/gated_lora.py:1-8): in round 0, whose verify row 0 sees
    only the prompt and itself, that row's logits are the base model's with or without adapters, while the
    proposal rows (1 on) move."""
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    cfg = shape_config("plm-tiny")
    base = PLMWeights.random(cfg, seed=9).with_ptp(rank=64, seed=10, projections=())
    full = PLMWeights.random(cfg, seed=9).with_ptp(rank=64, seed=10)
    prompt = torch.randint(0, cfg.vocab, (33,), generator=torch.Generator().manual_seed(3)).pin_memory()
    out = []
    for weights in (base, full):
        decoder = RoundDecoder(weights, 7, block_size=16, kv_cache_bytes=64 << 20, max_model_len=512)
        decoder._fill_aux(0)
        decoder.handle.load_prompt(prompt)
        decoder.handle.prefill()
        decoder.handle.round0()
        decoder.check()
        out.append((decoder.verify_logits[0].clone(), decoder.proposal_argmax(decoder.width)))
        decoder.close()
    torch.testing.assert_close(out[0][0], out[1][0], rtol=0, atol=0)  # verify row 0: the base model only
    assert out[0][1][1:] != out[1][1][1:]  # proposal rows: the adapters moved them
