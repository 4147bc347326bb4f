"""End-to-end token agreement at the PLM-1.3B shape (BASELINE configs[2]'s recipe: 256-token random prompts, exact
match with Voronoi sampling, seeds 0, 1, 2).

Two measures, both reported (PLM_PARITY_REPORT):
  - free running: the GPU decodes with RoundDecoder.generate on its own logits, the oracle decodes the same request
    on its own (its torch forward on the GPU in fp32 with TF32 off; the Voronoi decode and the bookkeeping in numpy).
    One flipped near-tie parts the sequences for good, so this gives the first divergence more than a rate;
  - per round, teacher forced: from the GPU's state before each round, whether the oracle's round (on its own
    logits) confirms the same tokens as the GPU's. The same rate between two correct oracles, one summing in fp32 and
    one in float64, is the model's intrinsic agreement: a random 24-layer bf16 stack moves its logits by ~0.1 under
    any change of rounding order, and its logits are flat enough that such a move flips the Voronoi cell of a
    verify row now and then. The GPU must agree with the oracle about as often as the two oracles agree with each
    other.
PLM_AGREEMENT_TOKENS sets the continuation length (48 by default; the report uses 512).
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import model as omodel
from oracle import voronoi as ov

pytestmark = pytest.mark.gpu

TOKENS = int(os.environ.get("PLM_AGREEMENT_TOKENS", "48"))


@pytest.fixture(scope="module")
def pair():
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = shape_config("plm-1.3b")
    weights = PLMWeights.random(cfg, seed=0)
    decoder = RoundDecoder(weights, 7, block_size=16, kv_cache_bytes=1 << 30, max_model_len=256 + TOKENS + 128)
    decoder.prepare()
    shape = omodel.ModelShape(cfg.num_layers, cfg.hidden, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                              cfg.intermediate, cfg.vocab, cfg.aux_vocab, cfg.num_aux_tokens, cfg.rms_eps,
                              cfg.rope_theta, decoder.cos_sin.shape[0])
    table = decoder.table.float().cpu().numpy()
    yield decoder, weights, shape, table, cfg
    decoder.close()


def _oracle(decoder, weights, shape, table, cfg, aux, accumulate="float32"):
    model = omodel.OracleModel(shape, weights.named(), "bfloat16", 16, decoder.num_pages,
                               np.arange(decoder.num_pages), cos_sin=decoder.cos_sin, device="cuda",
                               accumulate=accumulate)
    return omodel.RoundOracle(model, table, 7, "nucleus", None,
                              ov.VoronoiConfig(cfg.top_m, cfg.shortlist, cfg.rounds, cfg.sweeps),
                              capacity=decoder.out.numel(), aux_stream=aux)


def _confirmed(oracle, state) -> list[int]:
    """The tokens the oracle's own round confirms from ``state`` (its KV cache already holds the context)."""
    oracle.state = state.copy()
    base = oracle.state.base
    oracle.round(lazy=True)
    return oracle.state.out[base:oracle.state.base].tolist()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_token_agreement_plm_1p3b(pair, seed):
    decoder, weights, shape, table, cfg = pair
    prompt = torch.randint(0, cfg.vocab, (256,), generator=torch.Generator().manual_seed(1000 + seed))

    # free running
    gpu = decoder.generate(prompt, TOKENS, seed=seed, stop_at_eos=False).token_ids
    decoder.check()
    aux = decoder.aux_buf.cpu().numpy().copy()  # the request's cells (generate drew them from `seed`)
    oracle = _oracle(decoder, weights, shape, table, cfg, aux)
    oracle.prefill(prompt.numpy())
    oracle.round0()
    while oracle.state.base < TOKENS:
        oracle.round(lazy=True)
    ref = oracle.state.out[:TOKENS]
    got = np.asarray(gpu, dtype=np.int64)
    free = float((got == ref).mean())
    first = int(np.argmax(got != ref)) if free < 1 else TOKENS
    del oracle

    # per round, teacher forced from the GPU's state: GPU vs fp32 oracle, and fp32 oracle vs float64 oracle
    from oracle import rounds as orounds

    o32 = _oracle(decoder, weights, shape, table, cfg, aux)
    o64 = _oracle(decoder, weights, shape, table, cfg, aux, accumulate="float64")
    def gpu_state():
        return orounds.RoundState(7, decoder.out.numel(), int(decoder.offset_t), int(decoder.base_t),
                                  int(decoder.anchor[0]), decoder.pending.cpu().numpy().copy(),
                                  decoder.out.cpu().numpy().copy())

    decoder.handle.set_stop(1 << 62)
    decoder.handle.load_prompt(prompt.pin_memory())
    decoder.handle.prefill()
    torch.cuda.synchronize()
    after_prefill = gpu_state()
    decoder.handle.round0()
    for o in (o32, o64):  # each oracle's own context: the prompt, then round 0 from the GPU's state
        o.prefill_forward(prompt.numpy())
        o.state = after_prefill.copy()
        o.round0_forward()
    gpu_agree = intrinsic = rounds = 0
    while int(decoder.base_t) < TOKENS:
        st = gpu_state()
        a32, a64 = _confirmed(o32, st), _confirmed(o64, st)
        decoder.handle.round()
        torch.cuda.synchronize()
        mine = decoder.out[st.base:int(decoder.base_t)].tolist()
        gpu_agree += mine == a32
        intrinsic += a64 == a32
        rounds += 1
    decoder.check()
    rate, base_rate = gpu_agree / rounds, intrinsic / rounds
    print(f"seed {seed}: free-running agreement {free:.3f} over {TOKENS} tokens (first divergence at {first}); "
          f"per-round agreement GPU/oracle {rate:.3f}, oracle fp32/float64 {base_rate:.3f} over {rounds} rounds")
    out_dir = os.environ.get("PLM_PARITY_REPORT")
    if out_dir:
        with open(os.path.join(out_dir, f"agreement_plm-1.3b_seed{seed}.json"), "w") as f:
            json.dump({"seed": seed, "tokens": TOKENS, "free_running_agreement": free, "first_divergence": first,
                       "rounds": rounds, "per_round_gpu_vs_oracle": rate, "per_round_oracle_f32_vs_f64": base_rate},
                      f)
    del o32, o64
    torch.cuda.empty_cache()
    assert rate >= base_rate - 0.2, "the GPU flips verify decisions far more often than rounding alone does"
