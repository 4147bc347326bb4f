"""Generates the golden fixtures of tests/golden/ from the reference itself (run in the build container only).

    python tests/golden/make_golden.py --reference /path/to/PLM-anon [--out tests/golden]

The reference (justuswill/PLM-anon) has no CPU round path and no test fixtures of its own, so the fixtures come from
running its own functions on the CPU:
  layout.json       plm.mask.round_layout and RoundMaskView for several round shapes;
  quota.npz         plm.iterate.quota on random weights;
  accept.npz        plm.decoder.nucleus_acceptance / floor_acceptance on seeded logits;
  epilogue.npz      RoundDecoder._epilogue (steady round bookkeeping) and _prologue (ids, aux cells, embeddings,
                    positions, slots), called unbound on CPU tensors with a stand-in ``self``;
  round0.npz        RoundDecoder._round0 (round 0's inputs and commit) called unbound with a stand-in ``self`` whose
                    forward, logits and verify decode return seeded values;
  voronoi.npz       Voronoi.assign through LogitVoronoiAuxiliary (plm/iterate.py, plm/auxiliary.py) with the Triton
                    kernels run by the Triton interpreter (TRITON_INTERPRET=1; autotuning bypassed with fixed launch
                    meta GROUP=8, BLOCK=32; the compiled argmin replaced by its eager implementation);
  llama.npz         the Llama forward of Hugging Face transformers (LlamaForCausalLM, eager attention, fp32) over a
                    prompt plus one round under the round mask, pinning the oracle's paged forward;
  drift.json        how far a bf16 run of Hugging Face's LlamaForCausalLM (the reference's model family, in bf16
                    weights and bf16 arithmetic) lands from the oracle's forward (bf16 storage, fp32 sums) at the
                    PLM-1.3B shape on seeded random weights: the spread between two correct bf16 implementations of
                    the same model, which bounds the logit tolerance the GPU forward is held to;
  ptp.npz           the PTP scheme of the gated-LoRA model: LinearInterpolationAuxiliary.embed / decode_unmasked
                    (plm/auxiliary.py) and GatedLoraMethod.apply under gated_lora.rows_from (plm/gated_lora.py; its
                    GEMMs are vLLM's default unquantized GEMM, torch.nn.functional.linear, on the CPU).
Inputs that are large (logits rows, cost tables, model weights) are regenerated from the stored seeds by torch's CPU
generator, which is deterministic across machines; fixtures store their checksums so tests can confirm.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


# ---------------------------------------------------------------- shared input recipes (also used by the tests)
def voronoi_inputs(seed: int, n_rows: int, vocab: int, aux: int, kind: str):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(n_rows, vocab, generator=g) * 2.0
    if kind == "bf16":
        logits = logits.bfloat16().float()
    table = (torch.randn(vocab, aux, generator=g) * 0.3).bfloat16()
    return logits, table


def epilogue_logits(case: int, width: int, vocab: int):
    g = torch.Generator().manual_seed(4000 + case)
    return (torch.randn(width, vocab, generator=g) * 2).bfloat16().float()


def accept_inputs(seed: int, n_rows: int, vocab: int):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n_rows, vocab, generator=g) * 2.0).bfloat16().float()


def llama_weights(seed: int, layers: int, hidden: int, heads: int, kv_heads: int, head_dim: int, inter: int,
                  vocab: int):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g) * 0.02  # noqa: E731
    q_size, kv_size = heads * head_dim, kv_heads * head_dim
    w = {"embed": r(vocab + 1, hidden), "lm_head": r(vocab, hidden), "final_norm": 1 + r(hidden),
         "aux_vocab": r(64, hidden), "mask_aux": r(hidden), "qkv": [], "o": [], "gate_up": [], "down": [],
         "input_norm": [], "post_norm": []}
    for _ in range(layers):
        w["qkv"].append(r(q_size + 2 * kv_size, hidden))
        w["o"].append(r(hidden, q_size))
        w["gate_up"].append(r(2 * inter, hidden))
        w["down"].append(r(hidden, inter))
        w["input_norm"].append(1 + r(hidden))
        w["post_norm"].append(1 + r(hidden))
    return w


LLAMA = dict(seed=11, layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, inter=512, vocab=512)
DRIFT = {  # name -> shape; the tests look a case up by (shape name, layers)
    "plm-1.3b": dict(seed=13, layers=24, hidden=2048, heads=16, kv_heads=16, head_dim=128, inter=8192, vocab=50257,
                     prompt=64),
    "plm-3b_2layers": dict(seed=14, layers=2, hidden=2560, heads=20, kv_heads=20, head_dim=128, inter=10240,
                           vocab=50257, prompt=64),
}
VORONOI_CASES = [  # seed, rows, vocab, aux, kind
    (100, 2, 50257, 1024, "fp32"), (101, 2, 50257, 1024, "bf16"), (102, 3, 3000, 256, "fp32"),
    (103, 2, 8000, 512, "bf16"),
]
ACCEPT_CASES = [(200, 6, 50257), (201, 6, 4096)]


PTP_EMBED = (500, 24, 32, 3)                 # seed, values, hidden, embedding rows
PTP_DECODE = ((510, 16, 300, 16), (511, 16, 300, 128), (512, 4, 1000, 128))  # seed, rows, vocab, top_k
PTP_GATED = ((520, "float32"), (521, "bfloat16"))  # seed, dtype; shapes in ptp_gated_inputs
PTP_GATED_SHAPE = dict(rows=10, rows_from=3, d_in=64, shards=(48, 16, 16), rank=8)


def ptp_embed_inputs(seed: int, n: int, hidden: int, rows: int):
    g = torch.Generator().manual_seed(seed)
    table = torch.randn(rows, hidden, generator=g)
    values = torch.rand(n, generator=g)
    values[:6] = torch.tensor([0.0, 0.25, 0.5, 0.75, 1e-8, 0.99999994])
    return table, values


def ptp_decode_inputs(seed: int, n: int, vocab: int):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, vocab, generator=g) * 3.0).bfloat16().float(), torch.rand(n, generator=g)


def ptp_gated_inputs(seed: int, dtype: str):
    sh = PTP_GATED_SHAPE
    g = torch.Generator().manual_seed(seed)
    dt = getattr(torch, dtype)
    n_out = sum(sh["shards"])
    x = torch.randn(sh["rows"], sh["d_in"], generator=g).to(dt)
    weight = (torch.randn(n_out, sh["d_in"], generator=g) * 0.05).to(dt)
    lora_a = (torch.randn(len(sh["shards"]) * sh["rank"], sh["d_in"], generator=g) * 0.1).to(dt)
    lora_bs = [(torch.randn(w, sh["rank"], generator=g) * 0.1).to(dt) for w in sh["shards"]]
    return x, weight, lora_a, lora_bs


def checksum(t: torch.Tensor) -> float:
    return float(t.double().abs().sum())


# ---------------------------------------------------------------- generators
def gen_layout(ref, out: Path):
    from plm.mask import RoundMask, round_layout

    cases = {}
    for blocks in ([4] * 4, [6] * 6, [7] * 7, [8] * 8, [10] * 10, [55], [41], [1, 2, 3]):
        rel_positions, rel_aux, depth, own = round_layout(blocks, torch.device("cpu"))
        w = depth.numel()
        mask = RoundMask(w, torch.device("cpu"))
        mask.depth[:w].copy_(depth)
        mask.own_start[:w].copy_(own)
        offset = 37
        mask.offset.fill_(offset)
        q = torch.arange(offset, offset + w)[:, None]
        kv = torch.arange(0, offset + w)[None, :]
        visible = mask.view(torch.zeros(1), torch.zeros(1), q, kv)
        cases[",".join(map(str, blocks))] = {
            "rel_positions": rel_positions.tolist(), "rel_aux": rel_aux.tolist(), "depth": depth.tolist(),
            "own_start": own.tolist(), "offset": offset,
            "visible_rows": ["".join("1" if v else "0" for v in row) for row in visible.tolist()]}
    (out / "layout.json").write_text(json.dumps(cases))


def gen_quota(ref, out: Path):
    from plm.iterate import quota

    g = torch.Generator().manual_seed(300)
    weights = torch.rand(16, 128, generator=g) ** 4
    weights = weights / weights.sum(-1, keepdim=True)
    totals = [1024, 256, 4096, 7]
    counts = np.stack([quota(weights, t).numpy() for t in totals])
    np.savez_compressed(out / "quota.npz", weights=weights.numpy(), totals=np.asarray(totals), counts=counts)


def gen_accept(ref, out: Path):
    from plm.decoder import floor_acceptance, nucleus_acceptance

    rows = {}
    for seed, n, vocab in ACCEPT_CASES:
        logits = accept_inputs(seed, n, vocab)
        order = torch.argsort(logits, dim=-1, descending=True)
        ranks = torch.tensor([0, 1, 4, 30, 300, 3000])[:n]
        pending = order[torch.arange(n), ranks]
        res = {}
        for name, fn, thr in (("nucleus_0.94", nucleus_acceptance, 0.94), ("nucleus_0.5", nucleus_acceptance, 0.5),
                              ("exact", nucleus_acceptance, -1.0), ("floor_2e-3", floor_acceptance, 2e-3),
                              ("floor_1e-4", floor_acceptance, 1e-4)):
            res[name] = fn(logits, pending, torch.tensor(thr, dtype=torch.float32)).numpy()
        rows[f"{seed}"] = {"pending": pending.numpy(), "checksum": checksum(logits), **res}
    flat = {f"{seed}/{key}": np.asarray(value) for seed, d in rows.items() for key, value in d.items()}
    np.savez_compressed(out / "accept.npz", **flat)


def gen_epilogue(ref, out: Path):
    """RoundDecoder._prologue / _epilogue of plm/decoder.py, unbound, on CPU tensors."""
    from plm.auxiliary import LogitVoronoiAuxiliary
    from plm.decoder import RoundDecoder
    from plm.mask import round_layout

    records = {}
    g = torch.Generator().manual_seed(400)
    k, vocab, hidden, aux, bs = 7, 50257, 64, 1024, 16
    width = k + k * k
    scheme = LogitVoronoiAuxiliary(aux, hidden, vocab)
    scheme.auxiliary_vocabulary.copy_(torch.randn(aux, hidden, generator=g))
    scheme.mask_auxiliary.data.copy_(torch.randn(hidden, generator=g))
    embed_weight = torch.randn(vocab + 1, hidden, generator=g)
    for case, (nc_target, rule, thr) in enumerate([(0, "nucleus", -1.0), (3, "nucleus", -1.0), (6, "nucleus", -1.0),
                                                   (2, "nucleus", 0.94), (1, "floor", 2e-3)]):
        fake = types.SimpleNamespace(k=k, width=width, block_size=bs, vocab=vocab, sentinel=aux, num_aux_tokens=1,
                                     scheme=scheme, accept_rule=rule, sequence_capacity=64)
        logits = epilogue_logits(case, width, vocab)
        verify = torch.randint(0, vocab, (k,), generator=g)
        pending = torch.where(torch.arange(k - 1) < nc_target, verify[: k - 1], (verify[: k - 1] + 1) % vocab)
        anchor = torch.tensor([123])
        out_t = torch.full((512,), -1, dtype=torch.long)
        out_t[:40] = torch.arange(40)
        base_t = torch.tensor(40)
        offset_t = torch.tensor(300)
        round_sequence = torch.zeros(64, dtype=torch.long)
        sequence_step = torch.tensor([5])
        aux_buf = torch.randint(0, aux, (8192,), generator=g)
        rel_positions, rel_aux, _, _ = round_layout([k] * k, torch.device("cpu"))
        ids = torch.empty(width, dtype=torch.long)
        seq_lens, decode_offset = torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.int32)
        slot_mapping, kv_num_blocks = torch.zeros(width, dtype=torch.long), torch.zeros(1, dtype=torch.int32)
        mask_offset = torch.zeros((), dtype=torch.long)
        embeds, positions = RoundDecoder._prologue(
            fake, offset_t, base_t, anchor, pending.clone(), aux_buf, rel_positions, rel_aux, ids, mask_offset,
            seq_lens, decode_offset, slot_mapping, kv_num_blocks, torch.arange(width), embed_weight)
        pre = {"ids": ids.clone(), "positions": positions, "slot_mapping": slot_mapping.clone(),
               "embeds_checksum": np.float64(checksum(embeds)), "seq_lens": seq_lens.clone(),
               "kv_num_blocks": kv_num_blocks.clone()}
        pend = pending.clone()
        RoundDecoder._epilogue(fake, logits, verify, pend, anchor, out_t, base_t, offset_t, torch.arange(k),
                               torch.tensor(thr, dtype=torch.float32), torch.ones(1, dtype=torch.long), round_sequence,
                               sequence_step)
        post = {"out": out_t, "base": base_t, "offset": offset_t, "anchor": anchor, "pending": pend,
                "round_sequence": round_sequence, "sequence_step": sequence_step}
        inputs = {"logits_checksum": np.float64(checksum(logits)), "verify": verify, "pending_in": pending,
                  "aux_buf": aux_buf, "rule": torch.tensor(0 if rule == "nucleus" else 1),
                  "threshold": torch.tensor(thr)}
        for key, value in {**pre, **post, **inputs}.items():
            records[f"{case}/{key}"] = value.numpy() if isinstance(value, torch.Tensor) else np.asarray(value)
    records["embed_weight_checksum"] = np.asarray(checksum(embed_weight))
    np.savez_compressed(out / "epilogue.npz", **records)


ROUND0_CASES = ((600, 7, 45), (601, 4, 300), (602, 6, 1))  # seed, k, prompt length


def gen_round0(ref, out: Path):
    """RoundDecoder._round0 of plm/decoder.py, unbound, with the model calls stubbed by seeded values."""
    from plm.decoder import RoundDecoder
    from plm.mask import round_layout

    records = {}
    vocab, bs = 50257, 16
    for seed, k, prompt_len in ROUND0_CASES:
        width = k + k * k
        logits, verify_token, first, aux_buf = round0_inputs(seed, k, vocab)
        seen = {}

        def embed(ids, aux_values):
            seen["ids"], seen["aux_values"] = ids.clone(), aux_values.clone()
            return torch.zeros(ids.numel(), 4)

        def forward(md, slot_mapping, num_tokens, positions, embeds, gated_from=None):
            seen["positions"], seen["slot_mapping"], seen["gated_from"] = positions.clone(), slot_mapping.clone(), gated_from
            return torch.zeros(num_tokens, 4)

        def decode_verify(lg, hidden, index):
            seen["verify_index"] = index.clone()
            return verify_token.clone()

        fake = types.SimpleNamespace(
            k=k, width=width, block_size=bs, vocab=vocab, sentinel=1024, device=torch.device("cpu"),
            offset_t=torch.tensor(999), base_t=torch.tensor(999), out=torch.full((64,), 5, dtype=torch.long),
            prompt_len_t=torch.tensor(prompt_len), first=first.clone(), anchor=torch.tensor([7]),
            pending=torch.full((k - 1,), 9, dtype=torch.long), round0_layout=round_layout([width - 1], torch.device("cpu")),
            steady_layout=round_layout([k] * k, torch.device("cpu")), _install_tables=lambda layout: None,
            mask=types.SimpleNamespace(offset=torch.zeros((), dtype=torch.long)), ids_buf=torch.empty(width, dtype=torch.long),
            aux_buf=aux_buf, _embed=embed, seq_lens=torch.zeros(1, dtype=torch.int32),
            md=types.SimpleNamespace(decode_offset=torch.zeros(1, dtype=torch.int32)),
            slot_mapping=torch.zeros(width, dtype=torch.long), rows=torch.arange(width),
            kv_num_blocks=torch.zeros(1, dtype=torch.int32), _forward=forward,
            model=types.SimpleNamespace(compute_logits=lambda h: logits), _decode_verify=decode_verify,
            kidx=torch.arange(k))
        RoundDecoder._round0(fake)
        rec = {"out": fake.out, "base": fake.base_t, "offset": fake.offset_t, "anchor": fake.anchor,
               "pending": fake.pending, "first": first, "verify_token": verify_token,
               "inputs_checksum": np.float64(checksum(logits[:, :vocab]) + checksum(aux_buf)), "ids": seen["ids"],
               "aux_values": seen["aux_values"], "positions": seen["positions"], "slot_mapping": seen["slot_mapping"],
               "gated_from": torch.tensor(seen["gated_from"]), "verify_index": seen["verify_index"],
               "seq_lens": fake.seq_lens, "kv_num_blocks": fake.kv_num_blocks}
        for key, value in rec.items():
            records[f"{seed}/{key}"] = value.numpy() if isinstance(value, torch.Tensor) else np.asarray(value)
    np.savez_compressed(out / "round0.npz", **records)


def round0_inputs(seed: int, k: int, vocab: int = 50257):
    """gen_round0's seeded stand-ins: logits at compute_logits' padded width (cut to the vocabulary by _round0),
    the verify decode's token, the prefill's first token and the auxiliary stream."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(k + k * k, vocab + 7, generator=g)
    verify_token = torch.randint(0, vocab, (1,), generator=g)
    first = torch.randint(0, vocab, (1,), generator=g)
    aux_buf = torch.randint(0, 1024, (8192,), generator=g)
    return logits, verify_token, first, aux_buf


def gen_voronoi(ref, out: Path):
    import plm.iterate as it
    from plm.auxiliary import LogitVoronoiAuxiliary

    class Fixed:
        def __init__(self, fn, **meta):
            self.fn, self.meta = fn, meta

        def __getitem__(self, grid):
            return lambda *a, **kw: self.fn[grid](*a, **{**self.meta, **kw})

    it._scan_kernel = Fixed(it._scan_kernel.fn, GROUP=8, num_warps=4)
    it._condense_kernel = Fixed(it._condense_kernel.fn, BLOCK=32, num_warps=4)
    it._fused_argmin = it._argmin_impl
    records = {}
    for seed, n, vocab, aux, kind in VORONOI_CASES:
        logits, table = voronoi_inputs(seed, n, vocab, aux, kind)
        engine = it.Voronoi.from_table(table)
        a = engine.assign(logits, n_targets=128, k=8, rounds=2, iterations=12)
        cells = torch.randint(0, aux, (n,), generator=torch.Generator().manual_seed(seed + 1))
        scheme = LogitVoronoiAuxiliary(aux, 8, vocab)
        scheme._engine, scheme._cached_key = engine, None
        decoded = a.tokens.gather(1, a.sigma.gather(1, cells[:, None])).squeeze(1)
        key = f"{seed}"
        records.update({f"{key}/tokens": a.tokens.numpy(), f"{key}/counts": a.counts.numpy(),
                        f"{key}/sigma": a.sigma.numpy().astype(np.int16), f"{key}/bias": a.bias.numpy(),
                        f"{key}/cells": cells.numpy(), f"{key}/decoded": decoded.numpy(),
                        f"{key}/logits_checksum": np.asarray(checksum(logits)),
                        f"{key}/table_checksum": np.asarray(checksum(table.float()))})
        print(f"voronoi case {seed}: done", flush=True)
    np.savez_compressed(out / "voronoi.npz", **records)


def gen_llama(ref, out: Path):
    """HF LlamaForCausalLM (fp32, eager attention) on [prompt + one round] under the round mask."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from plm.mask import RoundMask, round_layout

    c = LLAMA
    w = llama_weights(c["seed"], c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"],
                      c["vocab"])
    cfg = LlamaConfig(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"],
                      num_hidden_layers=c["layers"], num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"],
                      head_dim=c["head_dim"], rms_norm_eps=1e-5, max_position_embeddings=4096,
                      tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    cfg._attn_implementation = "eager"
    model = LlamaForCausalLM(cfg).eval()
    q_size, kv_size = c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(w["embed"][: c["vocab"]])
        model.lm_head.weight.copy_(w["lm_head"])
        model.model.norm.weight.copy_(w["final_norm"])
        for i, layer in enumerate(model.model.layers):
            q, k, v = w["qkv"][i].split([q_size, kv_size, kv_size])
            layer.self_attn.q_proj.weight.copy_(q)
            layer.self_attn.k_proj.weight.copy_(k)
            layer.self_attn.v_proj.weight.copy_(v)
            layer.self_attn.o_proj.weight.copy_(w["o"][i])
            gate, up = w["gate_up"][i].split([c["inter"], c["inter"]])
            layer.mlp.gate_proj.weight.copy_(gate)
            layer.mlp.up_proj.weight.copy_(up)
            layer.mlp.down_proj.weight.copy_(w["down"][i])
            layer.input_layernorm.weight.copy_(w["input_norm"][i])
            layer.post_attention_layernorm.weight.copy_(w["post_norm"][i])
    k_round, prompt_len = 4, 24
    rel_positions, _, depth, own = (t.numpy() for t in round_layout([k_round] * k_round, torch.device("cpu")))
    width = rel_positions.size
    round_mask = RoundMask(width, torch.device("cpu"))
    round_mask.depth[:width].copy_(torch.as_tensor(depth))
    round_mask.own_start[:width].copy_(torch.as_tensor(own))
    round_mask.offset.fill_(prompt_len)
    g = torch.Generator().manual_seed(c["seed"] + 1)
    embeds = torch.randn(prompt_len + width, c["hidden"], generator=g) * 0.02
    total = prompt_len + width
    allowed = np.zeros((total, total), dtype=bool)
    allowed[:prompt_len, :prompt_len] = np.tril(np.ones((prompt_len, prompt_len), dtype=bool))
    q_idx = torch.arange(prompt_len, total)[:, None]
    kv_idx = torch.arange(total)[None, :]
    allowed[prompt_len:, :] = round_mask.view(None, None, q_idx, kv_idx).numpy()
    mask = torch.where(torch.as_tensor(allowed), 0.0, torch.finfo(torch.float32).min)[None, None]
    positions = torch.as_tensor(np.concatenate([np.arange(prompt_len), prompt_len + rel_positions]))[None]
    with torch.no_grad():
        logits = model(inputs_embeds=embeds[None], attention_mask=mask, position_ids=positions).logits[0]
    np.savez_compressed(out / "llama.npz", logits=logits.numpy(), embeds=embeds.numpy(), k=k_round,
                        prompt_len=prompt_len, **{f"cfg_{key}": value for key, value in c.items()})


def _hf_llama(c: dict, w: dict, dtype: torch.dtype):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"],
                      num_hidden_layers=c["layers"], num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"],
                      head_dim=c["head_dim"], rms_norm_eps=1e-5, max_position_embeddings=4096,
                      tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    cfg._attn_implementation = "eager"
    model = LlamaForCausalLM(cfg).eval()
    q_size, kv_size = c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(w["embed"][: c["vocab"]])
        model.lm_head.weight.copy_(w["lm_head"])
        model.model.norm.weight.copy_(w["final_norm"])
        for i, layer in enumerate(model.model.layers):
            q, k, v = w["qkv"][i].split([q_size, kv_size, kv_size])
            layer.self_attn.q_proj.weight.copy_(q)
            layer.self_attn.k_proj.weight.copy_(k)
            layer.self_attn.v_proj.weight.copy_(v)
            layer.self_attn.o_proj.weight.copy_(w["o"][i])
            gate, up = w["gate_up"][i].split([c["inter"], c["inter"]])
            layer.mlp.gate_proj.weight.copy_(gate)
            layer.mlp.up_proj.weight.copy_(up)
            layer.mlp.down_proj.weight.copy_(w["down"][i])
            layer.input_layernorm.weight.copy_(w["input_norm"][i])
            layer.post_attention_layernorm.weight.copy_(w["post_norm"][i])
    return model.to(dtype)


def gen_drift(ref, out: Path):
    """The bf16 drift of the reference's model family at the benchmark shapes: HF LlamaForCausalLM with bf16
    weights run (a) in bf16 and (b) in fp32, against the oracle's forward of the same weights (bf16 storage, fp32
    sums) and the oracle with float64 sums, over a causal prompt. Stores the max abs differences of the logits."""
    sys.path.insert(0, str(HERE.parent.parent))
    from oracle import model as omodel
    from oracle import rounds as orounds

    torch.set_num_threads(os.cpu_count() or 1)
    cases = {}
    for name, c in DRIFT.items():
        w = llama_weights(c["seed"], c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"],
                          c["vocab"])
        w = {key: ([t.bfloat16().float() for t in v] if isinstance(v, list) else v.bfloat16().float())
             for key, v in w.items()}
        ids = torch.randint(0, c["vocab"], (c["prompt"],), generator=torch.Generator().manual_seed(c["seed"] + 1))
        positions = torch.arange(c["prompt"])[None]
        logits = {}
        for kind, dtype in (("hf_bf16", torch.bfloat16), ("hf_fp32", torch.float32)):
            model = _hf_llama(c, w, dtype)
            with torch.no_grad():
                logits[kind] = model(input_ids=ids[None], position_ids=positions).logits[0].float()
            del model
        shape = omodel.ModelShape(c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["inter"],
                                  c["vocab"], 64, 1, 1e-5, 10000.0, 4096)
        pages = -(-c["prompt"] // 16)
        for kind, acc in (("oracle", "float32"), ("oracle_f64", "float64")):
            om = omodel.OracleModel(shape, w, "bfloat16", 16, pages, np.arange(pages), accumulate=acc)
            _, _, depth, own = orounds.chunk_layout(c["prompt"])
            embeds = om.embed_rows(ids.numpy(), np.full(c["prompt"], 64))
            hidden = om.forward(embeds, np.arange(c["prompt"]), 0, depth, own)
            logits[kind] = om.logits(hidden)
            del om
        diff = lambda a, b: float((logits[a] - logits[b]).abs().max())  # noqa: E731
        cases[name] = {"config": c, "logit_abs_max": float(logits["hf_fp32"].abs().max()),
                       "hf_bf16_vs_hf_fp32": diff("hf_bf16", "hf_fp32"),
                       "hf_bf16_vs_oracle": diff("hf_bf16", "oracle"), "hf_fp32_vs_oracle": diff("hf_fp32", "oracle"),
                       "oracle_vs_oracle_f64": diff("oracle", "oracle_f64")}
    res = {"cases": cases,
           "note": "max abs difference of the logits over all prompt rows; weights N(0, 0.02) rounded to bf16"}
    (out / "drift.json").write_text(json.dumps(res, indent=1) + "\n")


def gen_ptp(ref, out: Path):
    from plm import gated_lora
    from plm.auxiliary import LinearInterpolationAuxiliary

    res = {}
    seed, n, hidden, rows = PTP_EMBED
    table, values = ptp_embed_inputs(seed, n, hidden, rows)
    scheme = LinearInterpolationAuxiliary(hidden_size=hidden, text_vocab_size=100, num_embeddings=rows, top_k=16)
    with torch.no_grad():
        scheme.embedding.weight.copy_(table)
        ids = torch.full((n,), 100, dtype=torch.long)
        res["embed/out"] = scheme.embed(ids, values, ids == 100).numpy()
    res["embed/checksum"] = np.asarray(checksum(table) + checksum(values))
    for seed, n, vocab, top_k in PTP_DECODE:
        logits, u = ptp_decode_inputs(seed, n, vocab)
        scheme = LinearInterpolationAuxiliary(hidden_size=8, text_vocab_size=vocab, top_k=top_k)
        res[f"decode/{seed}/tokens"] = scheme.decode_unmasked(logits, None, None, u).numpy()
        res[f"decode/{seed}/checksum"] = np.asarray(checksum(logits) + checksum(u))

    class PlainLinear:  # the wrapped layer's own linear method
        def apply(self, layer, x, bias=None):
            return torch.nn.functional.linear(x, layer.weight, bias)

    for seed, dtype in PTP_GATED:
        x, weight, lora_a, lora_bs = ptp_gated_inputs(seed, dtype)
        layer = torch.nn.Module()
        layer.weight = torch.nn.Parameter(weight, requires_grad=False)
        layer.register_buffer("lora_a", lora_a, persistent=False)
        method = gated_lora.GatedLoraMethod(PlainLinear(), lora_bs)
        with torch.no_grad(), gated_lora.rows_from(PTP_GATED_SHAPE["rows_from"]):
            res[f"gated/{seed}/out"] = method.apply(layer, x).float().numpy()
        with torch.no_grad(), gated_lora.rows_from(None):
            res[f"gated/{seed}/ungated"] = method.apply(layer, x).float().numpy()
        res[f"gated/{seed}/checksum"] = np.asarray(checksum(x.float()) + checksum(weight.float()))
    np.savez_compressed(out / "ptp.npz", **res)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", required=True, help="checkout of justuswill/PLM-anon")
    parser.add_argument("--out", default=str(HERE))
    parser.add_argument("--only", nargs="*", default=None)
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    gens = {"layout": gen_layout, "quota": gen_quota, "accept": gen_accept, "epilogue": gen_epilogue,
            "voronoi": gen_voronoi, "llama": gen_llama, "ptp": gen_ptp, "round0": gen_round0, "drift": gen_drift}
    for name, fn in gens.items():
        if args.only is None or name in args.only:
            fn(args.reference, out)
            print(f"{name}: written", flush=True)


if __name__ == "__main__":
    main()
