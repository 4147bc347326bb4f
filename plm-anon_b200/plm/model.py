"""PLM model configuration and weights on the GPU.

A PLM export (plm/model.py:29-36 and plm/config.py of the reference) is a Llama checkpoint plus the auxiliary
scheme: ``config.json`` with Llama fields, ``text_vocab_size``, ``num_aux_tokens`` and an ``auxiliary_scheme`` dict
(plm/auxiliary.py:116-125), and safetensors with the Hugging Face Llama names and ``auxiliary_scheme.*``.
``PLMWeights`` holds the tensors the kernels read: q/k/v fused into one [(h + 2 kvh) * hd, d] matrix and gate/up
into one [2 I, d] matrix (vLLM's QKVParallelLinear / MergedColumnParallelLinear layout), in the model dtype.

Synthetic models (no checkpoints are available here) draw every matrix from N(0, 0.02) with a seeded generator in a
fixed order; ``save_export`` writes such a model as a loadable export directory.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16}


@dataclass
class PLMConfig:
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int = 50257            # text vocabulary (the logits the round reads)
    aux_vocab: int = 1024         # auxiliary_vocab_size A
    num_aux_tokens: int = 1
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_pos: int = 8192
    top_m: int = 128
    shortlist: int = 8
    rounds: int = 2
    sweeps: int = 12
    dtype: str = "bfloat16"
    name: str = "plm"

    @property
    def vocab_rows(self) -> int:
        """Embedding rows: the text vocabulary plus the auxiliary placeholder ids."""
        return self.vocab + self.num_aux_tokens

    def hf_config(self) -> dict:
        return {
            "architectures": ["PLMForCausalLM"], "model_type": "plm",
            "hidden_size": self.hidden, "intermediate_size": self.intermediate,
            "num_attention_heads": self.num_heads, "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim, "num_hidden_layers": self.num_layers, "rms_norm_eps": self.rms_eps,
            "rope_theta": self.rope_theta, "max_position_embeddings": self.max_pos, "hidden_act": "silu",
            "vocab_size": self.vocab_rows, "text_vocab_size": self.vocab, "num_aux_tokens": self.num_aux_tokens,
            "tie_word_embeddings": False, "torch_dtype": self.dtype,
            "auxiliary_scheme": {"kind": "logit_voronoi", "auxiliary_vocab_size": self.aux_vocab, "top_m": self.top_m,
                                 "iterate_shortlist": self.shortlist, "iterate_rounds": self.rounds,
                                 "iterate_sweeps": self.sweeps},
        }

    @classmethod
    def from_hf_config(cls, cfg: dict, name: str = "plm") -> "PLMConfig":
        scheme = cfg.get("auxiliary_scheme", {})
        if scheme.get("kind", "logit_voronoi") != "logit_voronoi":
            raise ValueError(f"unsupported auxiliary scheme {scheme.get('kind')!r} (only logit_voronoi)")
        heads = cfg["num_attention_heads"]
        rope = cfg.get("rope_theta", (cfg.get("rope_parameters") or {}).get("rope_theta", 10000.0))
        return cls(num_layers=cfg["num_hidden_layers"], hidden=cfg["hidden_size"], num_heads=heads,
                   num_kv_heads=cfg.get("num_key_value_heads", heads),
                   head_dim=cfg.get("head_dim", cfg["hidden_size"] // heads), intermediate=cfg["intermediate_size"],
                   vocab=cfg.get("text_vocab_size", cfg["vocab_size"]),
                   aux_vocab=scheme.get("auxiliary_vocab_size", 1024), num_aux_tokens=cfg.get("num_aux_tokens", 1),
                   rms_eps=cfg.get("rms_norm_eps", 1e-5), rope_theta=float(rope),
                   max_pos=cfg.get("max_position_embeddings", 8192), top_m=scheme.get("top_m", 128),
                   shortlist=scheme.get("iterate_shortlist", 8), rounds=scheme.get("iterate_rounds", 2),
                   sweeps=scheme.get("iterate_sweeps", 12), dtype=cfg.get("torch_dtype", "bfloat16"), name=name)


# Model shapes of the benchmark configurations (Llama family, SiLU-gated MLP, MHA).
SHAPES = {
    "plm-80m": dict(num_layers=12, hidden=512, num_heads=8, num_kv_heads=8, head_dim=64, intermediate=2048),
    "plm-1.3b": dict(num_layers=24, hidden=2048, num_heads=16, num_kv_heads=16, head_dim=128, intermediate=8192),
    "plm-3b": dict(num_layers=32, hidden=2560, num_heads=20, num_kv_heads=20, head_dim=128, intermediate=10240),
    "plm-tiny": dict(num_layers=2, hidden=256, num_heads=2, num_kv_heads=2, head_dim=128, intermediate=512),
}


def shape_config(name: str, **overrides) -> PLMConfig:
    return PLMConfig(**{**SHAPES[name], "name": name, **overrides})


def rope_cache(head_dim: int, max_pos: int, theta: float, dtype: torch.dtype) -> torch.Tensor:
    """[max_pos, head_dim]: cos | sin in fp32, cast to the model dtype (vLLM RotaryEmbedding's cos_sin_cache)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).to(dtype)


@dataclass
class PLMWeights:
    config: PLMConfig
    embed: torch.Tensor
    lm_head: torch.Tensor
    final_norm: torch.Tensor
    aux_vocab: torch.Tensor
    mask_aux: torch.Tensor
    qkv: list = field(default_factory=list)
    o: list = field(default_factory=list)
    gate_up: list = field(default_factory=list)
    down: list = field(default_factory=list)
    input_norm: list = field(default_factory=list)
    post_norm: list = field(default_factory=list)
    # The PTP scheme of the gated-LoRA model (plm/auxiliary.py:78-113, plm/gated_lora.py:35-90); None: the
    # logit-Voronoi scheme of every PLM. adapters: per layer, projection name -> (A [shards * rank][in],
    # B [out][rank] with the shards' up-projections stacked in output order).
    ptp_embedding: torch.Tensor | None = None
    ptp_top_k: int = 128
    adapters: list | None = None

    @property
    def device(self) -> torch.device:
        return self.embed.device

    @classmethod
    def random(cls, config: PLMConfig, seed: int = 0, device: str | torch.device = "cuda") -> "PLMWeights":
        """Seeded synthetic weights: matrices N(0, 0.02), norm weights 1 + N(0, 0.02), drawn in a fixed order."""
        dtype = DTYPES[config.dtype]
        g = torch.Generator(device=device).manual_seed(seed)
        c = config

        def mat(*shape, std=0.02, mean=0.0):
            t = torch.empty(*shape, device=device, dtype=torch.float32)
            t.normal_(mean, std, generator=g)
            return t.to(dtype)

        q_size, kv_size = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
        w = cls(config=c, embed=mat(c.vocab_rows, c.hidden), lm_head=mat(c.vocab, c.hidden),
                final_norm=mat(c.hidden, mean=1.0), aux_vocab=mat(c.aux_vocab, c.hidden), mask_aux=mat(c.hidden))
        for _ in range(c.num_layers):
            w.qkv.append(mat(q_size + 2 * kv_size, c.hidden))
            w.o.append(mat(c.hidden, q_size))
            w.gate_up.append(mat(2 * c.intermediate, c.hidden))
            w.down.append(mat(c.hidden, c.intermediate))
            w.input_norm.append(mat(c.hidden, mean=1.0))
            w.post_norm.append(mat(c.hidden, mean=1.0))
        return w

    def with_ptp(self, rank: int = 64, num_embeddings: int = 3, top_k: int = 128, seed: int = 0,
                 projections=("qkv", "o", "gate_up", "down")) -> "PLMWeights":
        """The same base model as a synthetic PTP model: a float32 interpolation table [num_embeddings, hidden] and
        rank-``rank`` adapters on ``projections`` of every layer, all N(0, 0.02) from a seeded generator."""
        c = self.config
        g = torch.Generator(device=self.device).manual_seed(seed)

        def mat(*shape, dtype):
            t = torch.empty(*shape, device=self.device, dtype=torch.float32)
            t.normal_(0.0, 0.02, generator=g)
            return t.to(dtype)

        q_size, kv_size = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
        shapes = {"qkv": (3, c.hidden, q_size + 2 * kv_size), "o": (1, q_size, c.hidden),
                  "gate_up": (2, c.hidden, 2 * c.intermediate), "down": (1, c.intermediate, c.hidden)}
        dtype = self.embed.dtype
        self.ptp_embedding = mat(num_embeddings, c.hidden, dtype=torch.float32)
        self.ptp_top_k = top_k
        self.adapters = [{name: (mat(shapes[name][0] * rank, shapes[name][1], dtype=dtype),
                                 mat(shapes[name][2], rank, dtype=dtype)) for name in projections}
                         for _ in range(c.num_layers)]
        return self

    def adapter_shards(self, layer: int, name: str) -> list[int]:
        """Output widths of a projection's shards, in output order (q, k, v; gate, up)."""
        c = self.config
        q_size, kv_size = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
        return {"qkv": [q_size, kv_size, kv_size], "o": [c.hidden], "gate_up": [c.intermediate, c.intermediate],
                "down": [c.hidden]}[name]

    def named(self) -> dict:
        """Tensors by name for the CPU oracle (lists per layer)."""
        return {"embed": self.embed, "lm_head": self.lm_head, "final_norm": self.final_norm,
                "aux_vocab": self.aux_vocab, "mask_aux": self.mask_aux, "qkv": self.qkv, "o": self.o,
                "gate_up": self.gate_up, "down": self.down, "input_norm": self.input_norm,
                "post_norm": self.post_norm}

    # ---------------------------------------------------------------- export directory (HF Llama names)
    def save_export(self, directory: str | Path) -> Path:
        from safetensors.torch import save_file

        c = self.config
        out = Path(directory)
        out.mkdir(parents=True, exist_ok=True)
        q_size, kv_size = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
        tensors = {"model.embed_tokens.weight": self.embed, "lm_head.weight": self.lm_head,
                   "model.norm.weight": self.final_norm,
                   "auxiliary_scheme.auxiliary_vocabulary": self.aux_vocab,
                   "auxiliary_scheme.mask_auxiliary": self.mask_aux}
        for i in range(c.num_layers):
            p = f"model.layers.{i}."
            q, k, v = self.qkv[i].split([q_size, kv_size, kv_size])
            gate, up = self.gate_up[i].split([c.intermediate, c.intermediate])
            tensors.update({p + "self_attn.q_proj.weight": q, p + "self_attn.k_proj.weight": k,
                            p + "self_attn.v_proj.weight": v, p + "self_attn.o_proj.weight": self.o[i],
                            p + "mlp.gate_proj.weight": gate, p + "mlp.up_proj.weight": up,
                            p + "mlp.down_proj.weight": self.down[i], p + "input_layernorm.weight": self.input_norm[i],
                            p + "post_attention_layernorm.weight": self.post_norm[i]})
        save_file({name: t.contiguous().cpu() for name, t in tensors.items()}, str(out / "model.safetensors"))
        (out / "config.json").write_text(json.dumps(c.hf_config(), indent=1))
        return out

    @classmethod
    def from_export(cls, directory: str | Path, device: str | torch.device = "cuda",
                    dtype: str | None = None) -> "PLMWeights":
        """Load an export in its own ``torch_dtype``, or converted to ``dtype`` when one is given (the conversion
        is recorded in ``config.dtype``; nothing is reinterpreted)."""
        from safetensors import safe_open

        directory = Path(directory)
        cfg = json.loads((directory / "config.json").read_text())
        if "PLMForCausalLM" not in cfg.get("architectures", []):
            raise ValueError(f"{directory} is not a PLM export (architectures {cfg.get('architectures')})")
        c = PLMConfig.from_hf_config(cfg, name=directory.name)
        if dtype is not None:
            c.dtype = dtype
        dtype = DTYPES.get(c.dtype)
        if dtype is None:
            raise ValueError(f"model dtype {c.dtype} is not supported (bfloat16 or float16)")
        tensors = {}
        for shard in sorted(directory.glob("*.safetensors")):
            with safe_open(str(shard), "pt") as handle:
                for name in handle.keys():
                    tensors[name] = handle.get_tensor(name)

        def get(name):
            if name not in tensors:
                raise KeyError(f"{name} is missing from {directory}")
            return tensors[name].to(device=device, dtype=dtype).contiguous()

        lm = tensors.get("lm_head.weight", tensors.get("model.embed_tokens.weight"))
        w = cls(config=c, embed=get("model.embed_tokens.weight"),
                lm_head=lm[: c.vocab].to(device=device, dtype=dtype).contiguous(), final_norm=get("model.norm.weight"),
                aux_vocab=get("auxiliary_scheme.auxiliary_vocabulary"),
                mask_aux=get("auxiliary_scheme.mask_auxiliary"))
        for i in range(c.num_layers):
            p = f"model.layers.{i}."
            w.qkv.append(torch.cat([get(p + "self_attn.q_proj.weight"), get(p + "self_attn.k_proj.weight"),
                                    get(p + "self_attn.v_proj.weight")]).contiguous())
            w.o.append(get(p + "self_attn.o_proj.weight"))
            w.gate_up.append(torch.cat([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")]).contiguous())
            w.down.append(get(p + "mlp.down_proj.weight"))
            w.input_norm.append(get(p + "input_layernorm.weight"))
            w.post_norm.append(get(p + "post_attention_layernorm.weight"))
        return w


def config_dict(config: PLMConfig) -> dict:
    return asdict(config)
