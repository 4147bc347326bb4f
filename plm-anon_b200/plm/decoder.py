"""Parallel decoding rounds on libplm_native.so (same interface as the reference's plm/decoder.py).

One request at a time. A round decodes ``W = k + k*k`` query positions: ``k`` verify rows and ``k`` proposal
blocks of ``k`` rows. All loop-carried state lives on the device inside the native handle, so a steady round is
one CUDA-graph replay of ``plm_round`` (forward, lm_head, verify decode, acceptance and commit all in kernels),
followed by a non-blocking copy of ``base`` and the first output tokens into pinned memory — the reference's
hot loop (plm/decoder.py:312-324, 414-447) without vLLM, FlexAttention, Triton or torch.compile.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch

from . import native
from .model import PLMWeights, rope_cache

AUX_STREAM_LENGTH = 8192  # plm/decoder.py:28
EOS_WINDOW = 1024         # plm/decoder.py:29


@dataclass
class DecodeResult:
    token_ids: list[int]
    text: str
    seconds: float
    steady_rounds: int
    steady_ms: float
    steady_tokens: int

    @property
    def tokens_per_second(self) -> float:
        return len(self.token_ids) / self.seconds if self.seconds else 0.0


class RoundDecoder:
    """Drop-in for plm.decoder.RoundDecoder over the native round engine.

    ``accept_rule`` is ``nucleus`` (``threshold`` None: exact match) or ``floor``. ``block_size`` is the KV page
    size; ``kv_cache_bytes`` sizes the page pool; ``block_table`` optionally maps logical to physical pages
    (default identity). ``separate_mlp`` runs gate_up and down as two launches instead of the one persistent MLP
    block launch (for comparison; forwards wider than 128 rows always use two)."""

    sequence_capacity = 1 << 17

    def __init__(self, weights: PLMWeights, k: int, accept_rule: str = "nucleus", threshold: float | None = None,
                 chunk_widths: tuple[int, ...] = (), *, block_size: int = 64, kv_cache_bytes: int = 1 << 30,
                 max_model_len: int = 4096, tokenizer=None, eos_token_id: int | None = None,
                 block_table: list[int] | None = None, max_prefill: int = 256, separate_mlp: bool = False) -> None:
        if accept_rule not in ("nucleus", "floor"):
            raise ValueError(f"accept rule {accept_rule!r}: nucleus or floor")
        if not torch.cuda.is_available():
            raise native.NativeError("RoundDecoder needs an sm_100a GPU; there is no CPU path")
        self.weights, self.config = weights, weights.config
        c = self.config
        self.k, self.width = k, k + k * k
        self.block_size = block_size
        self.accept_rule, self.threshold = accept_rule, threshold
        self.tokenizer, self.eos_token_id = tokenizer, eos_token_id
        if eos_token_id is None and tokenizer is not None:
            self.eos_token_id = tokenizer.eos_token_id
        self.max_model_len = max_model_len
        self.max_pages = -(-(max_model_len + 2 * self.width + block_size) // block_size)
        page_bytes = c.num_layers * 2 * c.num_kv_heads * block_size * c.head_dim * 2
        self.num_pages = max(self.max_pages, kv_cache_bytes // page_bytes)
        self.max_seq = self.max_pages * block_size
        self.cos_sin = rope_cache(c.head_dim, max(c.max_pos, self.max_seq), c.rope_theta,
                                  weights.embed.dtype).to(weights.device)
        self._layer_arrays = [(native.c_void_p * c.num_layers)(*[t.data_ptr() for t in getattr(weights, name)])
                              for name in ("qkv", "o", "gate_up", "down", "input_norm", "post_norm")]
        model = native.ModelDesc(
            dtype=native.PLM_BF16, num_layers=c.num_layers, hidden=c.hidden, num_heads=c.num_heads,
            num_kv_heads=c.num_kv_heads, head_dim=c.head_dim, intermediate=c.intermediate, vocab=c.vocab,
            aux_vocab=c.aux_vocab, num_aux_tokens=c.num_aux_tokens, rms_eps=c.rms_eps,
            max_pos=self.cos_sin.shape[0], top_m=c.top_m, shortlist=min(c.shortlist, c.top_m), rounds=c.rounds,
            sweeps=c.sweeps, epsilon=0.15, refocus=0.35, endpoint=0.0087)
        ptrs = native.WeightPtrs(
            embed=weights.embed.data_ptr(), lm_head=weights.lm_head.data_ptr(),
            final_norm=weights.final_norm.data_ptr(), aux_vocab=weights.aux_vocab.data_ptr(),
            mask_aux=weights.mask_aux.data_ptr(), cos_sin=self.cos_sin.data_ptr(),
            qkv=self._layer_arrays[0], o=self._layer_arrays[1], gate_up=self._layer_arrays[2],
            down=self._layer_arrays[3], input_norm=self._layer_arrays[4], post_norm=self._layer_arrays[5], table=None)
        rule = native.RULE_FLOOR if accept_rule == "floor" else native.RULE_NUCLEUS
        round_desc = native.RoundDesc(
            k=k, rule=rule, threshold=-1.0 if threshold is None else float(threshold), page_size=block_size,
            num_pages=self.num_pages, max_pages=self.max_pages, out_capacity=self.max_seq,
            seq_capacity=self.sequence_capacity, aux_len=AUX_STREAM_LENGTH, max_prefill=max_prefill,
            separate_mlp=1 if separate_mlp else 0)
        self.handle = native.Handle(model, ptrs, round_desc, keepalive=(weights, self.cos_sin, self._layer_arrays))
        if block_table is not None:
            self.handle.set_block_table(block_table)
        st = self.handle.state()
        self._state = st
        self.out = native.device_view(st.out, (st.out_capacity,), torch.int64)
        self.base_t = native.device_view(st.base, (), torch.int64)
        self.offset_t = native.device_view(st.offset, (), torch.int64)
        self.anchor = native.device_view(st.anchor, (1,), torch.int64)
        self.pending = native.device_view(st.pending, (k - 1,), torch.int64)
        self.round_sequence = native.device_view(st.round_sequence, (st.seq_capacity,), torch.int64)
        self.sequence_step = native.device_view(st.sequence_step, (1,), torch.int64)
        self.aux_buf = native.device_view(st.aux_buf, (st.aux_len,), torch.int64)
        self.verify_logits = native.device_view(st.verify_logits, (k, c.vocab), torch.float32)
        self.hidden_normed = native.device_view(st.hidden_normed, (st.row_capacity, c.hidden), torch.bfloat16)
        self.kv_cache = native.device_view(
            st.kv_cache, (c.num_layers, 2, self.num_pages, c.num_kv_heads, block_size, c.head_dim), torch.bfloat16)
        self.table = native.device_view(st.table, (c.vocab, c.aux_vocab), torch.bfloat16)
        self.base_host = torch.zeros((), dtype=torch.long).pin_memory()
        self.tokens_host = torch.empty(EOS_WINDOW, dtype=torch.long).pin_memory()
        self.aux_seed: int | None = None
        self.graph: torch.cuda.CUDAGraph | None = None

    # ------------------------------------------------------------------ construction
    def prepare(self) -> None:
        """Capture the steady round (plus the pinned-memory reads) into a CUDA graph."""
        self._fill_aux(0)
        # the capture runs the round twice eagerly on a benign state first (offset 0, base 1)
        self.offset_t.zero_()
        self.base_t.fill_(1)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(2):
                self._round_body()
        torch.cuda.current_stream().wait_stream(stream)
        self.handle.check()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._round_body()
        self.graph = graph
        torch.cuda.synchronize()
        self.handle.check()

    def _round_body(self) -> None:
        self.handle.round()
        self.base_host.copy_(self.base_t, non_blocking=True)
        self.tokens_host.copy_(self.out[:EOS_WINDOW], non_blocking=True)

    def _fill_aux(self, seed: int) -> None:
        """The request's auxiliary cell stream: randint(A) from a CUDA generator seeded with ``seed``
        (plm/decoder.py:407-412 with LogitVoronoiAuxiliary.sample_prior, plm/auxiliary.py:46-48)."""
        if self.aux_seed == seed:
            return
        generator = torch.Generator(device="cuda").manual_seed(seed)
        cells = torch.randint(self.config.aux_vocab, (AUX_STREAM_LENGTH,), device="cuda", generator=generator,
                              dtype=torch.long)
        self.handle.set_aux_stream(cells)
        torch.cuda.current_stream().synchronize()
        self.aux_seed = seed

    # ------------------------------------------------------------------ the request
    def _prompt_ids(self, prompt) -> torch.Tensor:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("a text prompt needs a tokenizer; pass token ids instead")
            prompt = self.tokenizer(prompt).input_ids
        ids = torch.as_tensor(prompt, dtype=torch.long).flatten()
        return ids.pin_memory() if not ids.is_cuda else ids

    def _replay_until_tokens(self, num_tokens: int) -> int:
        replays = 0
        while True:
            self.graph.replay()
            replays += 1
            event = torch.cuda.Event()
            event.record()
            event.synchronize()
            if int(self.base_host) >= num_tokens:
                return replays

    def _replay_until_eos_or_tokens(self, num_tokens: int) -> int:
        end_of_text, limit = self.eos_token_id, min(num_tokens, EOS_WINDOW)
        replays, seen = 0, 2  # round 0 confirms exactly one token, so base is 2 when the loop starts
        while True:
            self.graph.replay()
            replays += 1
            event = torch.cuda.Event()
            event.record()
            event.synchronize()
            base = int(self.base_host)
            if end_of_text in self.tokens_host[seen:min(base, limit)].tolist() or base >= num_tokens:
                return replays
            seen = base

    def _steady_loop(self, num_tokens: int, stop_at_eos: bool) -> tuple[int, float]:
        start_event, end_event = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start_event.record()
        if stop_at_eos and self.eos_token_id is not None:
            replays = self._replay_until_eos_or_tokens(num_tokens)
        else:
            replays = self._replay_until_tokens(num_tokens)
        end_event.record()
        torch.cuda.synchronize()
        return replays, start_event.elapsed_time(end_event)

    @torch.inference_mode()
    def generate(self, prompt, num_tokens: int, *, seed: int = 0, stop_at_eos: bool = True) -> DecodeResult:
        """Decode ``num_tokens`` tokens after ``prompt`` (text with a tokenizer, or token ids)."""
        if self.graph is None:
            self.prepare()
        torch.cuda.synchronize()
        started = time.perf_counter()
        ids = self._prompt_ids(prompt)
        length = ids.numel()
        if length + num_tokens + 2 * self.width + self.block_size > self.max_seq:
            raise ValueError(f"prompt ({length}) + tokens ({num_tokens}) exceeds max_model_len {self.max_seq} "
                             f"for width {self.width}")
        self._fill_aux(seed)
        self.handle.load_prompt(ids)
        self.handle.prefill()
        self.handle.round0()
        replays, steady_ms = self._steady_loop(num_tokens, stop_at_eos)
        seconds = time.perf_counter() - started
        tokens = self.out[:num_tokens].tolist()
        eos = self.eos_token_id
        if stop_at_eos and eos is not None and eos in tokens:
            tokens = tokens[: tokens.index(eos) + 1]
        final_base = int(self.base_t.item())
        text = self.tokenizer.decode(tokens) if self.tokenizer is not None else ""
        return DecodeResult(token_ids=tokens, text=text, seconds=seconds, steady_rounds=replays,
                            steady_ms=steady_ms, steady_tokens=final_base - 2)

    def proposal_argmax(self, rows: int) -> list[int]:
        """Argmax token (first index on ties) of forward rows [0, rows) from the lm_head's per-tile partials of the
        last round (rows with logits written in full are not reduced there: use ``verify_logits`` for those)."""
        st = self._state
        val = native.device_view(st.best_val, (st.lm_tiles, st.width), torch.float32)[:, :rows]
        idx = native.device_view(st.best_idx, (st.lm_tiles, st.width), torch.int32)[:, :rows]
        top = val.max(dim=0).values
        first = torch.where(val == top[None, :], idx, torch.full_like(idx, 1 << 30)).min(dim=0).values
        return first.long().tolist()

    def check(self) -> None:
        """Raise if any kernel recorded a device error (out-of-range index, timed-out wait)."""
        self.handle.check()

    def close(self) -> None:
        self.graph = None
        self.handle.close()


def pages_for(tokens: int, block_size: int) -> int:
    return math.ceil(tokens / block_size)
