"""Parallel decoding rounds on libplm_native.so (same interface as the reference's plm/decoder.py).

One request at a time. A round decodes ``W = k + k*k`` query positions: ``k`` verify rows and ``k`` proposal
blocks of ``k`` rows. All loop-carried state lives on the device inside the native handle, so a steady round is
one CUDA-graph replay of ``plm_round`` (forward, lm_head, verify decode, acceptance and commit all in kernels),
followed by a non-blocking copy of ``base`` and the done flag into pinned memory. The stop test (token budget,
end-of-text) of the reference's hot loop (plm/decoder.py:312-324, 414-447) runs on the device, so the host keeps
rounds queued instead of waiting for each one; no vLLM, FlexAttention, Triton or torch.compile is involved.
"""

from __future__ import annotations

import math
import time
from collections import deque
from dataclasses import dataclass

import torch

from . import native
from .model import PLMWeights, rope_cache

AUX_STREAM_LENGTH = 8192  # plm/decoder.py:28
EOS_WINDOW = 1024         # plm/decoder.py:29: end-of-text is looked for among the first EOS_WINDOW output positions
ROUNDS_IN_FLIGHT = 2      # steady-round replays queued ahead of the one the host waits for


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
                 block_table: list[int] | None = None, max_prefill: int = 256, separate_mlp: bool = False,
                 release_block_weights: bool = False) -> None:
        if accept_rule not in ("nucleus", "floor"):
            raise ValueError(f"accept rule {accept_rule!r}: nucleus or floor")
        if not torch.cuda.is_available():
            raise native.NativeError("RoundDecoder needs an sm_100a GPU; there is no CPU path")
        self.weights, self.config = weights, weights.config
        c = self.config
        stored = {t.dtype for t in [weights.embed, weights.lm_head, weights.aux_vocab, *weights.qkv, *weights.o,
                                     *weights.gate_up, *weights.down, *weights.input_norm, *weights.post_norm]}
        if len(stored) != 1 or not stored <= {torch.bfloat16, torch.float16}:
            raise native.NativeError(f"RoundDecoder: weights stored as {sorted(map(str, stored))}; the sm_100a kernels "
                                     "take one model dtype, bfloat16 or float16 (convert explicitly, e.g. "
                                     "RoundConfig(dtype='bfloat16') or PLMWeights.from_export(..., dtype=...))")
        self.dtype = stored.pop()
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
            dtype=native.PLM_F16 if self.dtype == torch.float16 else native.PLM_BF16, num_layers=c.num_layers, hidden=c.hidden, num_heads=c.num_heads,
            num_kv_heads=c.num_kv_heads, head_dim=c.head_dim, intermediate=c.intermediate, vocab=c.vocab,
            aux_vocab=c.aux_vocab, num_aux_tokens=c.num_aux_tokens, rms_eps=c.rms_eps,
            max_pos=self.cos_sin.shape[0], top_m=c.top_m, shortlist=min(c.shortlist, c.top_m), rounds=c.rounds,
            sweeps=c.sweeps, epsilon=0.15, refocus=0.35, endpoint=0.0087)
        self.ptp = weights.ptp_embedding is not None
        ptp_desc = self._ptp_desc(weights) if self.ptp else None
        ptrs = native.WeightPtrs(
            embed=weights.embed.data_ptr(), lm_head=weights.lm_head.data_ptr(),
            final_norm=weights.final_norm.data_ptr(), aux_vocab=weights.aux_vocab.data_ptr(),
            mask_aux=weights.mask_aux.data_ptr(), cos_sin=self.cos_sin.data_ptr(),
            qkv=self._layer_arrays[0], o=self._layer_arrays[1], gate_up=self._layer_arrays[2],
            down=self._layer_arrays[3], input_norm=self._layer_arrays[4], post_norm=self._layer_arrays[5], table=None,
            ptp=None if ptp_desc is None else native.pointer(ptp_desc))
        rule = native.RULE_FLOOR if accept_rule == "floor" else native.RULE_NUCLEUS
        round_desc = native.RoundDesc(
            k=k, rule=rule, threshold=-1.0 if threshold is None else float(threshold), page_size=block_size,
            num_pages=self.num_pages, max_pages=self.max_pages, out_capacity=self.max_seq,
            seq_capacity=self.sequence_capacity, aux_len=AUX_STREAM_LENGTH, max_prefill=max_prefill,
            separate_mlp=1 if separate_mlp else 0)
        self.handle = native.Handle(model, ptrs, round_desc,
                                    keepalive=(weights, self.cos_sin, self._layer_arrays, ptp_desc))
        # A handle that reads only its packed copies of o, gate_up and down leaves the originals to the caller; with
        # release_block_weights (for weights this decoder owns, as RoundConfig.build's) they are dropped here.
        self.released_block_weights = False
        if release_block_weights and not (self.handle.borrowed_weights() & native.WEIGHTS_BLOCK):
            weights.o = weights.gate_up = weights.down = None
            self.released_block_weights = True
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
        self.hidden_normed = native.device_view(st.hidden_normed, (st.row_capacity, c.hidden), self.dtype)
        self.kv_cache = native.device_view(
            st.kv_cache, (c.num_layers, 2, self.num_pages, c.num_kv_heads, block_size, c.head_dim), self.dtype)
        self.table = None if self.ptp else native.device_view(st.table, (c.vocab, c.aux_vocab), self.dtype)
        self.stop_block = native.device_view(st.stop, (4,), torch.int64)
        # [base, done] of the newest finished round, copied by every replay into pinned host memory
        self.poll_host = torch.zeros(2, dtype=torch.long).pin_memory()
        self.aux_seed: int | None = None
        self.graph: torch.cuda.CUDAGraph | None = None

    # ------------------------------------------------------------------ construction
    def prepare(self) -> None:
        """Capture the steady round and its pinned-memory poll into one CUDA graph. The round runs twice eagerly
        first, from a harmless state (empty context, base 1, no stop), so every kernel has been loaded and tuned."""
        self._fill_aux(0)
        self.offset_t.zero_()
        self.base_t.fill_(1)
        self.handle.set_stop(1 << 62)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self._enqueue_round()
            self._enqueue_round()
        torch.cuda.current_stream().wait_stream(side)
        self.handle.check()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._enqueue_round()
        torch.cuda.synchronize()
        self.handle.check()
        self.graph = graph

    def _enqueue_round(self) -> None:
        self.handle.round()
        self.poll_host[0].copy_(self.base_t, non_blocking=True)
        self.poll_host[1].copy_(self.stop_block[3], non_blocking=True)

    def _ptp_desc(self, weights: PLMWeights) -> native.PtpDesc:
        """The PTP scheme for plm_create: the interpolation table and, per projection, arrays of per-layer A and B
        pointers (null where a layer's projection has no adapter)."""
        adapters = weights.adapters or []
        rank = adapters[0][next(iter(adapters[0]))][1].shape[1] if adapters and adapters[0] else 0
        arrays = {}
        for name in ("qkv", "o", "gate_up", "down"):
            for i, part in enumerate(("a", "b")):
                ptrs = [layer[name][i].data_ptr() if name in layer else None for layer in adapters]
                arrays[f"{name}_{part}"] = (native.c_void_p * len(ptrs))(*ptrs) if any(ptrs) else None
        self._ptp_arrays = arrays
        return native.PtpDesc(embedding=weights.ptp_embedding.data_ptr(), num_embeddings=weights.ptp_embedding.shape[0],
                              top_k=weights.ptp_top_k, rank=rank, **arrays)

    def _fill_aux(self, seed: int) -> None:
        """Per request: the auxiliary stream from a CUDA generator seeded with ``seed`` (plm/decoder.py:407-412), as
        the scheme's sample_prior draws it: A-ary cells for the logit-Voronoi scheme (plm/auxiliary.py:46-48),
        uniforms in [0, 1) for the PTP scheme (plm/auxiliary.py:92-94). A seed already in the handle is not drawn
        again."""
        if seed == self.aux_seed:
            return
        generator = torch.Generator(device="cuda").manual_seed(seed)
        if self.ptp:
            cells = torch.rand(AUX_STREAM_LENGTH, dtype=torch.float32, device="cuda", generator=generator)
            self.handle.set_aux_uniforms(cells)
        else:
            cells = torch.randint(self.config.aux_vocab, (AUX_STREAM_LENGTH,), dtype=torch.long, device="cuda",
                                  generator=generator)
            self.handle.set_aux_stream(cells)
        torch.cuda.current_stream().synchronize()  # ``cells`` must outlive the copy
        self.aux_seed = seed

    # ------------------------------------------------------------------ the request
    def _as_ids(self, prompt) -> torch.Tensor:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("a text prompt needs a tokenizer; pass token ids instead")
            prompt = self.tokenizer(prompt).input_ids
        ids = torch.as_tensor(prompt, dtype=torch.long).reshape(-1)
        return ids if ids.is_cuda else ids.pin_memory()

    def _decode_rounds(self) -> int:
        """Replay steady rounds until the device reports the request finished; return how many rounds committed.

        The stop test runs on the device, in the bookkeeping of the round that reaches the budget or confirms the
        end-of-text token, so the host never has to see a round before queuing the next: ``ROUNDS_IN_FLIGHT``
        replays stay queued, and the host only waits on the oldest. Replays queued behind the stopping round
        find the done flag and commit nothing, so the output equals the one-round-at-a-time loop's."""
        first_step = int(self.sequence_step.item())
        queued: deque[torch.cuda.Event] = deque()
        finished = False
        while not finished:
            while len(queued) < ROUNDS_IN_FLIGHT:
                self.graph.replay()
                marker = torch.cuda.Event()
                marker.record()
                queued.append(marker)
            queued.popleft().synchronize()
            finished = bool(self.poll_host[1])
        while queued:
            queued.popleft().synchronize()
        return int(self.sequence_step.item()) - first_step

    @torch.inference_mode()
    def generate(self, prompt, num_tokens: int, *, seed: int = 0, stop_at_eos: bool = True) -> DecodeResult:
        """Decode ``num_tokens`` tokens after ``prompt`` (text with a tokenizer, or token ids): prefill and first
        token, round 0, then steady rounds until the budget or, with ``stop_at_eos``, the end-of-text token."""
        if self.graph is None:
            self.prepare()
        torch.cuda.synchronize()
        t_request = time.perf_counter()
        ids = self._as_ids(prompt)
        needed = ids.numel() + num_tokens + 2 * self.width + self.block_size
        if needed > self.max_seq:
            raise ValueError(f"prompt ({ids.numel()}) + tokens ({num_tokens}) exceeds max_model_len {self.max_seq} "
                             f"for width {self.width}")
        eos = self.eos_token_id if stop_at_eos else None
        self._fill_aux(seed)
        self.handle.set_stop(num_tokens, eos, min(num_tokens, EOS_WINDOW))
        self.handle.load_prompt(ids)
        self.handle.prefill()
        self.handle.round0()
        t_steady, t_done = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_steady.record()
        rounds = self._decode_rounds()
        t_done.record()
        torch.cuda.synchronize()
        seconds = time.perf_counter() - t_request
        produced = self.out[:num_tokens].tolist()
        if eos is not None and eos in produced:
            produced = produced[: produced.index(eos) + 1]
        committed = int(self.base_t.item())  # round 0 leaves base at 2, so the steady rounds added committed - 2
        return DecodeResult(token_ids=produced,
                            text=self.tokenizer.decode(produced) if self.tokenizer is not None else "",
                            seconds=seconds, steady_rounds=rounds, steady_ms=t_steady.elapsed_time(t_done),
                            steady_tokens=committed - 2)

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
