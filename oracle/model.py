"""CPU restatement of the round's forward and state machine (test infrastructure).

The model is the Llama forward the reference runs through vLLM (vllm/model_executor/models/llama.py:81-314 as
installed; the PLM classes add only the auxiliary scheme, plm/model.py:29-36):
  layer:  residual add + RMSNorm (vllm ir/ops/layernorm.py: fp32 sum, stored rounded as the new residual,
          normalised unrounded, ``x.to(dtype) * weight``) -> fused qkv -> neox rotary embedding with the cos/sin
          cache of vllm rotary_embedding/base.py:69-96 (fp32, cast to the model dtype) -> attention over the paged
          KV cache under the round mask -> o_proj -> add + RMSNorm -> gate_up -> silu(gate) * up -> down_proj;
  head:   final add + RMSNorm, lm_head, logits rounded to the model dtype.
Tensors are float32 holding model-dtype values; every point where the GPU stores a tensor in the model dtype is
a rounding point here too (``_r``). The paged KV cache has the GPU's layout
[layer][K|V][page][kv_head][slot][head_dim] and is addressed through a block table.

RoundOracle strings the pieces into the RoundDecoder of plm/decoder.py: prefill (369-403, first token 384),
round 0 (275-310) and steady rounds (312-365), with the verify decode of ``oracle.voronoi`` and the bookkeeping of
``oracle.rounds``. Given a ``ptp.PTPScheme`` (and optionally adapters) the model is instead the gated-LoRA PTP model
of ``oracle.ptp``: blended auxiliary inputs, adapters on the gated rows and the inverse-CDF verify decode.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import ptp as optp
from . import rounds as orounds
from . import voronoi as ov

TORCH_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


@dataclass
class ModelShape:
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int            # text vocabulary (logits width)
    aux_vocab: int
    num_aux_tokens: int = 1
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_pos: int = 8192


def rope_cache(head_dim: int, max_pos: int, theta: float, dtype: torch.dtype) -> torch.Tensor:
    """[max_pos, head_dim]: cos | sin, computed in fp32 and cast to the model dtype (vllm base.py:69-96)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(dtype)


class OracleModel:
    """Llama forward over a paged KV cache; ``weights`` maps the Llama / auxiliary-scheme names to CPU tensors."""

    def __init__(self, shape: ModelShape, weights: dict, dtype: str, page_size: int, num_pages: int,
                 block_table: np.ndarray, cos_sin: torch.Tensor | None = None, accumulate: str = "float32",
                 ptp: "optp.PTPScheme | None" = None, adapters: "list[dict] | None" = None,
                 device: str | torch.device = "cpu"):
        """``accumulate="float64"`` runs every matmul and attention product in double precision (then rounds to
        float32): the same model with another summation order, to measure how far rounding alone moves the output.
        ``ptp``: the linear-interpolation scheme replaces the logit-Voronoi auxiliary inputs; ``adapters``: per layer,
        projection name ("qkv", "o", "gate_up", "down") -> ``optp.Adapter``, applied on the gated rows. ``device``:
        where the torch arithmetic runs (the CPU by default; a checker on a GPU box may put it on a GPU, with TF32
        off, to follow long free-running decodes)."""
        self.s, self.dtype, self.tdtype = shape, dtype, TORCH_DTYPES[dtype]
        self.acc = torch.float64 if accumulate == "float64" else torch.float32
        self.device = torch.device(device)
        f = lambda t: t.detach().to(self.device, torch.float32)  # noqa: E731
        self.embed = f(weights["embed"])
        self.lm_head = f(weights["lm_head"])[: shape.vocab]
        self.final_norm = f(weights["final_norm"])
        self.aux_vocab = f(weights["aux_vocab"])
        self.mask_aux = f(weights["mask_aux"])
        self.layers = [{name: f(weights[name][i]) for name in ("qkv", "o", "gate_up", "down", "input_norm",
                                                                "post_norm")} for i in range(shape.num_layers)]
        if cos_sin is None:
            cos_sin = rope_cache(shape.head_dim, shape.max_pos, shape.rope_theta, self.tdtype)
        self.cos_sin = f(cos_sin)
        self.page_size, self.num_pages = page_size, num_pages
        self.block_table = np.asarray(block_table, dtype=np.int64)
        self.kv = torch.zeros(shape.num_layers, 2, num_pages, shape.num_kv_heads, page_size, shape.head_dim,
                              device=self.device)
        self.ptp = ptp
        self.adapters = adapters if adapters is not None else [{} for _ in range(shape.num_layers)]

    # ------------------------------------------------------------------ helpers
    def _r(self, x: torch.Tensor) -> torch.Tensor:
        """Round to the model dtype and back (a stored tensor)."""
        return x.to(self.tdtype).to(torch.float32)

    def _mm(self, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return (a.to(self.acc) @ b.to(self.acc)).to(torch.float32)

    def _einsum(self, spec: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        return torch.einsum(spec, a.to(self.acc), b.to(self.acc)).to(torch.float32)

    def _rmsnorm(self, x32: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        variance = x32.pow(2).mean(dim=-1, keepdim=True)
        return self._r(self._r(x32 * torch.rsqrt(variance + self.s.rms_eps)) * weight)

    def slots(self, logical: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        pages = self.block_table[logical // self.page_size]
        return pages, logical % self.page_size

    def embed_rows(self, ids: np.ndarray, aux_values: np.ndarray) -> torch.Tensor:
        """plm/decoder.py:264-268 with LogitVoronoiAuxiliary.embed (plm/auxiliary.py:50-54), or with the PTP
        scheme's blend cast to the model dtype."""
        V, A = self.s.vocab, self.s.aux_vocab
        ids = torch.as_tensor(ids, dtype=torch.int64, device=self.device)
        aux_mask = (ids >= V) & (ids < V + self.s.num_aux_tokens)
        token = self.embed[ids.masked_fill(aux_mask, 0).clamp(0, V - 1)]
        if self.ptp is not None:
            blend = optp.linear_interpolation_embed(np.asarray(aux_values, dtype=np.float32), self.ptp.embedding)
            return torch.where(aux_mask[:, None], self._r(torch.from_numpy(blend).to(self.device)), token)
        values = torch.as_tensor(aux_values, dtype=torch.int64, device=self.device)
        vectors = self.aux_vocab[values.clamp(max=A - 1).clamp(min=0)]
        vectors = torch.where((values == A)[:, None], self.mask_aux[None, :], vectors)
        return torch.where(aux_mask[:, None], vectors, token)

    def _proj(self, index: int, name: str, x: torch.Tensor, gated_from: int | None) -> torch.Tensor:
        """One projection of layer ``index`` in the model dtype, with its adapters on the gated rows."""
        weight = self.layers[index][name]
        return optp.gated_projection(x, weight, self.adapters[index].get(name), gated_from, self._r, self._mm)

    # ------------------------------------------------------------------ forward
    def forward(self, embeds: torch.Tensor, positions: np.ndarray, offset: int, depth: np.ndarray,
                own_start: np.ndarray, gated_from: int | None = None) -> torch.Tensor:
        """Rows at logical KV indices offset + r; writes their K/V into the cache; returns the final-norm output.
        ``gated_from``: the first row the adapters apply to (None: none)."""
        s = self.s
        rows, hd = embeds.shape[0], s.head_dim
        half = hd // 2
        q_size, kv_size = s.num_heads * hd, s.num_kv_heads * hd
        dev = self.device
        pos = torch.as_tensor(positions, dtype=torch.int64, device=dev)
        cos, sin = self.cos_sin[pos, :half][:, None, :], self.cos_sin[pos, half:][:, None, :]
        n_keys = offset + rows
        mask = torch.as_tensor(orounds.visible(np.asarray(depth), np.asarray(own_start), offset, n_keys), device=dev)
        logical = np.arange(n_keys, dtype=np.int64)
        key_pages, key_slots = (torch.as_tensor(a, device=dev) for a in self.slots(logical))
        row_pages, row_slots = (torch.as_tensor(a, device=dev)
                                for a in self.slots(offset + np.arange(rows, dtype=np.int64)))
        group = s.num_heads // s.num_kv_heads

        residual = embeds.clone()
        x = self._rmsnorm(residual, self.layers[0]["input_norm"])
        for index, layer in enumerate(self.layers):
            qkv = self._proj(index, "qkv", x, gated_from)
            q = qkv[:, :q_size].view(rows, s.num_heads, hd)
            k = qkv[:, q_size:q_size + kv_size].view(rows, s.num_kv_heads, hd)
            v = qkv[:, q_size + kv_size:].view(rows, s.num_kv_heads, hd)

            def rope(t):
                x1, x2 = t[..., :half], t[..., half:]
                return self._r(torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1))

            q, k = rope(q), rope(k)
            self.kv[index, 0, row_pages, :, row_slots, :] = k
            self.kv[index, 1, row_pages, :, row_slots, :] = v
            keys = self.kv[index, 0, key_pages, :, key_slots, :]     # [n_keys, kv_heads, hd]
            values = self.kv[index, 1, key_pages, :, key_slots, :]
            keys = keys.repeat_interleave(group, dim=1)
            values = values.repeat_interleave(group, dim=1)
            scores = self._einsum("rhd,khd->hrk", q, keys) / math.sqrt(hd)
            scores = scores.masked_fill(~mask[None], float("-inf"))
            probs = torch.softmax(scores, dim=-1)
            attn = self._r(self._einsum("hrk,khd->rhd", probs, values).reshape(rows, q_size))
            y = self._proj(index, "o", attn, gated_from)
            summed = y + residual
            residual = self._r(summed)
            x = self._rmsnorm(summed, layer["post_norm"])
            gu = self._proj(index, "gate_up", x, gated_from)
            gate, up = gu[:, : s.intermediate], gu[:, s.intermediate:]
            act = self._r(gate / (1.0 + torch.exp(-gate)) * up)
            y = self._proj(index, "down", act, gated_from)
            summed = y + residual
            residual = self._r(summed)
            weight = self.layers[index + 1]["input_norm"] if index + 1 < len(self.layers) else self.final_norm
            x = self._rmsnorm(summed, weight)
        return x

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """compute_logits -> [:, :vocab] in the model dtype (plm/decoder.py:318), as fp32 values."""
        return self._r(self._mm(hidden, self.lm_head.T))


class RoundOracle:
    """The RoundDecoder state machine (plm/decoder.py:85-467) on the CPU oracle model."""

    def __init__(self, model: OracleModel, table: np.ndarray, k: int, rule: str = "nucleus",
                 threshold: float | None = None, config: ov.VoronoiConfig = ov.VoronoiConfig(),
                 capacity: int = 4096, aux_stream: np.ndarray | None = None):
        self.model, self.k, self.width = model, k, k + k * k
        self.table = None if table is None else np.asarray(table, dtype=np.float32)  # unused by the PTP scheme
        self.rule, self.threshold = rule, (-1.0 if threshold is None else float(threshold))
        self.config = config
        self.state = orounds.RoundState(k, capacity)
        self.ptp = model.ptp
        # the PTP scheme streams uniforms and gives non-auxiliary rows the value 0 (plm/decoder.py:107-108, 137)
        stream_dtype = np.float32 if self.ptp is not None else np.int64
        self.sentinel = 0 if self.ptp is not None else model.s.aux_vocab
        self.aux = np.zeros(orounds.AUX_STREAM_LENGTH, dtype=stream_dtype) if aux_stream is None else aux_stream
        self.steady = orounds.steady_layout(k)
        self.r0 = orounds.round0_layout(k)
        self.last_logits = None
        self.last_hidden = None

    def decode(self, logits_row: np.ndarray, value) -> int:
        """The verify decode of one row: the Voronoi cell's token, or the PTP scheme's inverse CDF at u."""
        if self.ptp is not None:
            return optp.icdf_decode_row(logits_row, float(value), self.ptp.top_k)
        return ov.decode_row(logits_row, self.table, int(value), self.model.dtype, self.config).token

    # ---- forward halves (write KV, return the final-norm hidden rows and their logits) ----
    def prefill_forward(self, prompt: np.ndarray, chunk: int = 256):
        """Causal prefill in chunks (plm/decoder.py:369-403); returns (hidden, logits) of the last prompt row."""
        prompt = np.asarray(prompt, dtype=np.int64)
        n, sentinel = prompt.size, self.sentinel
        for start in range(0, n, chunk):
            rows = min(chunk, n - start)
            _, _, depth, own = orounds.chunk_layout(rows)
            embeds = self.model.embed_rows(prompt[start:start + rows], np.full(rows, sentinel))
            hidden = self.model.forward(embeds, start + np.arange(rows), start, depth, own)
        last = hidden[n - 1 - start: n - start]
        return last, self.model.logits(last).cpu().numpy()

    def round0_forward(self):
        st, layout = self.state, self.r0
        ids, values, positions, _ = orounds.round0_prologue(st, layout, self.model.s.vocab, self.sentinel, self.aux)
        hidden = self.model.forward(self.model.embed_rows(ids, values), positions, st.offset, layout[2], layout[3],
                                    gated_from=1)
        return hidden, self.model.logits(hidden).cpu().numpy()

    def round_forward(self):
        st, layout = self.state, self.steady
        ids, values, positions, _ = orounds.prologue(st, layout, self.model.s.vocab, self.sentinel, self.aux)
        hidden = self.model.forward(self.model.embed_rows(ids, values), positions, st.offset, layout[2], layout[3],
                                    gated_from=self.k)
        return hidden, self.model.logits(hidden).cpu().numpy()

    # ---- commits (acceptance / bookkeeping on given logits) ----
    def commit_first(self, logits_row: np.ndarray, prompt_len: int) -> int:
        first = self.decode(logits_row, self.aux[0])
        orounds.first_token(self.state, first, prompt_len)
        return first

    def commit_round0(self, verify_logits: np.ndarray, proposal_argmax: np.ndarray) -> int:
        """``proposal_argmax``: argmax of rows 1..W-1 (plm/decoder.py:300-306)."""
        verify0 = self.decode(verify_logits[0], self.aux[self.state.base])
        orounds.round0_epilogue(self.state, verify0, proposal_argmax)
        return verify0

    def commit_round(self, verify_logits: np.ndarray, proposal_argmax: np.ndarray, lazy: bool = False) -> int:
        """``verify_logits``: the k verify rows; ``proposal_argmax``: argmax of the k^2 proposal rows. ``lazy``
        decodes the verify rows in order only up to the first one that rejects its proposal: the rows after it
        never reach the output or the state (plm/decoder.py:351-365 reads verify[nc] and the proposals before
        it), so the round's result is the same and the decode costs nc + 1 rows instead of k."""
        st, k = self.state, self.k
        verify = np.full(k, -1, dtype=np.int64)
        rule = np.zeros(k, dtype=bool)
        for d in range(k):
            verify[d] = self.decode(verify_logits[d], self.aux[st.base + d])
            if d < k - 1:
                if self.rule == "floor":
                    rule[d] = ov.floor_accepts(verify_logits[d], int(st.pending[d]), self.threshold)
                else:
                    rule[d] = ov.nucleus_accepts(verify_logits[d], int(st.pending[d]), self.threshold)
                if lazy and not (verify[d] == st.pending[d] or rule[d]):
                    break
        return orounds.epilogue(st, verify, rule, proposal_argmax)

    # ---- whole steps on the oracle's own logits ----
    def prefill(self, prompt: np.ndarray, chunk: int = 256) -> int:
        hidden, logits = self.prefill_forward(prompt, chunk)
        self.last_hidden, self.last_logits = hidden, logits
        return self.commit_first(logits[0], int(np.asarray(prompt).size))

    def round0(self) -> None:
        hidden, logits = self.round0_forward()
        self.last_hidden, self.last_logits = hidden, logits
        self.commit_round0(logits[:1], orounds.argmax_first(logits[1:]))

    def round(self, lazy: bool = False) -> int:
        hidden, logits = self.round_forward()
        self.last_hidden, self.last_logits = hidden, logits
        return self.commit_round(logits[: self.k], orounds.argmax_first(logits[self.k:]), lazy=lazy)
