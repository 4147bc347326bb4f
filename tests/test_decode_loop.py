"""The request loop of RoundDecoder.generate: the device-side stop test with rounds kept in flight must give exactly
what the reference's loop gives (plm/decoder.py:414-439: replay one round, wait for it, read base and the confirmed
tokens on the host, stop at the token budget or at end-of-text), and weights are never reinterpreted in another
dtype."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _decoder(k: int = 7, seed: int = 1):
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    weights = PLMWeights.random(shape_config("plm-tiny"), seed=seed)
    decoder = RoundDecoder(weights, k, block_size=16, kv_cache_bytes=64 << 20, max_model_len=1024)
    decoder.prepare()
    return decoder


def _one_round_at_a_time(decoder, prompt, num_tokens: int, seed: int, eos: int | None):
    """The reference's host loop on the same engine: the device never stops by itself; the host waits for every
    round, then tests the budget and the newly confirmed tokens below the end-of-text window."""
    decoder._fill_aux(seed)
    decoder.handle.set_stop(1 << 62)
    decoder.handle.load_prompt(torch.as_tensor(prompt, dtype=torch.long).pin_memory())
    decoder.handle.prefill()
    decoder.handle.round0()
    step0 = int(decoder.sequence_step.item())
    window = min(num_tokens, 1024)
    seen, rounds = 2, 0
    while True:
        decoder.handle.round()
        rounds += 1
        torch.cuda.synchronize()
        base = int(decoder.base_t.item())
        confirmed = decoder.out[seen:min(base, window)].tolist() if min(base, window) > seen else []
        if (eos is not None and eos in confirmed) or base >= num_tokens:
            break
        seen = base
    tokens = decoder.out[:num_tokens].tolist()
    if eos is not None and eos in tokens:
        tokens = tokens[: tokens.index(eos) + 1]
    record = decoder.round_sequence[step0:int(decoder.sequence_step.item())].tolist()
    return tokens, rounds, base - 2, record


@pytest.mark.parametrize("k,num_tokens", [(7, 40), (4, 33), (1, 9)])
def test_rounds_in_flight_match_one_at_a_time(k, num_tokens):
    decoder = _decoder(k)
    prompt = list(range(200, 264))
    ref_tokens, ref_rounds, ref_steady, ref_record = _one_round_at_a_time(decoder, prompt, num_tokens, 3, None)
    step0 = int(decoder.sequence_step.item())
    res = decoder.generate(prompt, num_tokens, seed=3, stop_at_eos=False)
    record = decoder.round_sequence[step0:int(decoder.sequence_step.item())].tolist()
    decoder.check()
    assert res.token_ids == ref_tokens
    assert (res.steady_rounds, res.steady_tokens) == (ref_rounds, ref_steady)
    assert record == ref_record, "rounds queued after the stop must commit nothing"
    assert int(decoder.stop_block[3]) == 1

    # end-of-text: a token the budget-only run confirmed in a steady round becomes the end-of-text id
    candidates = [t for p, t in enumerate(ref_tokens) if 4 <= p < len(ref_tokens) - 3 and t not in ref_tokens[:p]]
    if not candidates:
        pytest.skip("no token first confirmed in the middle of the continuation")
    eos = candidates[0]
    decoder.eos_token_id = eos
    ref = _one_round_at_a_time(decoder, prompt, num_tokens, 3, eos)
    step0 = int(decoder.sequence_step.item())
    res = decoder.generate(prompt, num_tokens, seed=3, stop_at_eos=True)
    record = decoder.round_sequence[step0:int(decoder.sequence_step.item())].tolist()
    decoder.check()
    assert res.token_ids == ref[0] and res.token_ids[-1] == eos
    assert (res.steady_rounds, res.steady_tokens, record) == (ref[1], ref[2], ref[3])
    decoder.close()


def test_float16_export_runs_in_float16(tmp_path):
    """A float16 export (the reference's default dtype, plm/rounds.py:50) builds and decodes in float16: the handle's
    model dtype is float16, and nothing is reinterpreted. Weights of mixed dtypes fail loudly. Converting the export
    explicitly (RoundConfig(dtype='bfloat16')) decodes the same tokens as a model built from the same values
    rounded to bfloat16."""
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config
    from plm.native import NativeError
    from plm.rounds import RoundConfig

    cfg = shape_config("plm-tiny", dtype="float16")
    weights = PLMWeights.random(cfg, seed=2)
    export = weights.save_export(tmp_path / "fp16")
    assert RoundConfig(model=str(export)).dtype == "float16"
    native16 = RoundConfig(model=str(export), max_model_len=1024).build(kv_cache_bytes=64 << 20, block_size=16)
    assert native16.dtype == torch.float16 and native16.handle.model.dtype == 1  # PLM_F16
    prompt = list(range(10, 50))
    t16 = native16.generate(prompt, 24, seed=1, stop_at_eos=False).token_ids
    native16.check()
    assert len(t16) == 24
    native16.close()

    mixed = PLMWeights.from_export(export)
    mixed.o = [t.bfloat16() for t in mixed.o]
    with pytest.raises(NativeError):
        RoundDecoder(mixed, 7, block_size=16, kv_cache_bytes=64 << 20)

    converted = RoundConfig(model=str(export), dtype="bfloat16", max_model_len=1024).build(kv_cache_bytes=64 << 20,
                                                                                          block_size=16)
    direct = PLMWeights.from_export(export)
    for name in ("qkv", "o", "gate_up", "down", "input_norm", "post_norm"):
        setattr(direct, name, [t.bfloat16() for t in getattr(direct, name)])
    for name in ("embed", "lm_head", "final_norm", "aux_vocab", "mask_aux"):
        setattr(direct, name, getattr(direct, name).bfloat16())
    same = RoundDecoder(direct, 7, block_size=16, kv_cache_bytes=64 << 20, max_model_len=1024)
    a = converted.generate(prompt, 24, seed=1, stop_at_eos=False).token_ids
    b = same.generate(prompt, 24, seed=1, stop_at_eos=False).token_ids
    assert a == b and len(a) == 24
    converted.close()
    same.close()


def test_released_block_weights_decode_the_same():
    """A decoder that frees its o, gate_up and down originals (the handle reads its packed copies everywhere, the
    separate GEMMs of a 200-row prefill chunk included) decodes bit for bit what one keeping them decodes, and the
    originals' memory is returned."""
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    cfg = shape_config("plm-tiny")
    keep = RoundDecoder(PLMWeights.random(cfg, seed=6), 7, block_size=16, kv_cache_bytes=64 << 20,
                        max_model_len=1024)
    assert not keep.released_block_weights
    weights = PLMWeights.random(cfg, seed=6)
    layer_bytes = sum(t.numel() * t.element_size() for t in [*weights.o, *weights.gate_up, *weights.down])
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    freed = RoundDecoder(weights, 7, block_size=16, kv_cache_bytes=64 << 20, max_model_len=1024,
                         release_block_weights=True)
    torch.cuda.synchronize()
    assert freed.released_block_weights and weights.o is None and weights.down is None
    assert torch.cuda.memory_allocated() - before <= -layer_bytes + (1 << 20) + _allocated_by(freed)
    prompt = torch.randint(0, cfg.vocab, (200,), generator=torch.Generator().manual_seed(2))
    results = []
    for decoder in (keep, freed):
        decoder._fill_aux(3)
        decoder.handle.set_stop(1 << 62)
        decoder.handle.load_prompt(prompt.pin_memory())
        decoder.handle.prefill()
        decoder.handle.round0()
        for _ in range(3):
            decoder.handle.round()
        torch.cuda.synchronize()
        decoder.check()
        results.append((decoder.out[:16].clone(), decoder.verify_logits.clone(), int(decoder.base_t)))
    assert torch.equal(results[0][0], results[1][0]) and results[0][2] == results[1][2]
    assert torch.equal(results[0][1], results[1][1])


def _allocated_by(decoder) -> int:
    """Bytes torch allocated for the decoder's own tensors (rotary table and pinned views are not device allocations
    beyond the rotary cache)."""
    return decoder.cos_sin.numel() * decoder.cos_sin.element_size()
