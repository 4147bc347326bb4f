"""The PLM decoding configuration behind ``--setting``, ``--mode``, ``--match`` and ``--k`` (same interface as the
reference's plm/rounds.py), and the round decoder it builds.

``--mode`` is accepted for drop-in compatibility: both ``fast`` and ``default`` run the same native sm_100a kernels
(the reference's ``fast`` patched Triton GEMM tiles into vLLM, ``default`` was stock vLLM). ``--match exact``
accepts a proposal only if it equals the verify row's own decode; ``--match relaxed`` also accepts proposals
passing the setting's looser rule: the top-0.94 nucleus for post-trained models, probability above 2e-3 for
pretrained ones.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

PREFILL_BUCKETS = tuple(range(64, 641, 64))  # plm/rounds.py:16


@dataclass(frozen=True)
class Setting:
    default_k: dict[str, int]
    relaxed_rule: tuple[str, float]


# plm/rounds.py:26-29
SETTINGS = {
    "posttrain": Setting(default_k={"exact": 7, "relaxed": 10}, relaxed_rule=("nucleus", 0.94)),
    "pretrain": Setting(default_k={"exact": 6, "relaxed": 6}, relaxed_rule=("floor", 2e-3)),
}


def is_plm_export(model: str) -> bool:
    config = Path(model) / "config.json"
    return config.exists() and "PLMForCausalLM" in json.loads(config.read_text()).get("architectures", [])


def export_dtype(model: str) -> str:
    """The ``torch_dtype`` an export directory declares (float16 when it declares none, the reference's default,
    plm/rounds.py:50)."""
    config = json.loads((Path(model) / "config.json").read_text())
    return str(config.get("torch_dtype", "float16"))


def scheme_kind(scheme: str) -> str | None:
    config = json.loads((Path(scheme) / "config.json").read_text())
    return config.get("auxiliary_scheme", {}).get("kind")


@dataclass
class RoundConfig:
    """``model`` is an export directory or ``synthetic:<shape>[:seed=<n>]`` (e.g. ``synthetic:plm-1.3b``).
    ``dtype`` None keeps the export's own ``torch_dtype`` (bfloat16 for synthetic models); naming one converts the
    weights explicitly. The kernels run bfloat16 and float16 (the reference's default, plm/rounds.py:50); any other
    dtype makes ``build`` raise ``NativeError``."""
    model: str
    setting: str = "posttrain"
    mode: str = "fast"
    match: str = "exact"
    k: int | None = None
    dtype: str | None = None
    max_model_len: int = 4096

    def __post_init__(self) -> None:
        if self.setting not in SETTINGS:
            raise ValueError(f"--setting {self.setting!r}: one of {tuple(SETTINGS)}")
        if self.match not in ("exact", "relaxed"):
            raise ValueError(f"--match {self.match!r}: exact or relaxed")
        if self.mode not in ("fast", "default"):
            raise ValueError(f"--mode {self.mode!r}: fast or default")
        if self.k is None:
            self.k = SETTINGS[self.setting].default_k[self.match]
        if self.dtype is None and self.model.startswith("synthetic:"):
            self.dtype = "bfloat16"
        elif self.dtype is None and (Path(self.model) / "config.json").exists():
            self.dtype = export_dtype(self.model)

    @property
    def accept(self) -> tuple[str, float | None]:
        """Exact match is the nucleus test switched off, in either setting (plm/rounds.py:57-60)."""
        return SETTINGS[self.setting].relaxed_rule if self.match == "relaxed" else ("nucleus", None)

    @property
    def width(self) -> int:
        return self.k + self.k * self.k

    def describe(self) -> dict:
        rule, threshold = self.accept
        return {"setting": self.setting, "mode": self.mode, "match": self.match, "k": self.k, "width": self.width,
                "dtype": self.dtype, "model": self.model,
                "accept": f"{rule} {threshold}" if threshold is not None else "exact", "engine": "plm-b200"}

    def weights(self):
        from .model import PLMWeights, shape_config

        if self.model.startswith("synthetic:"):
            parts = self.model.split(":")
            seed = 0
            for extra in parts[2:]:
                if extra.startswith("seed="):
                    seed = int(extra[5:])
            return PLMWeights.random(shape_config(parts[1], dtype=self.dtype), seed=seed)
        return PLMWeights.from_export(self.model, dtype=self.dtype)

    def build(self, gpu_memory_utilization: float = 0.25, kv_cache_bytes: int = 1 << 30, block_size: int = 64):
        """The prepared RoundDecoder (plm/rounds.py:71-81). ``gpu_memory_utilization`` is accepted for drop-in
        compatibility; the KV pool is sized by ``kv_cache_bytes``."""
        from .decoder import RoundDecoder
        from .native import NativeError

        if self.dtype not in ("bfloat16", "float16"):
            raise NativeError(f"dtype {self.dtype}: the native kernels are built for bfloat16 and float16")
        rule, threshold = self.accept
        tokenizer = None
        if not self.model.startswith("synthetic:"):
            try:
                from transformers import AutoTokenizer

                tokenizer = AutoTokenizer.from_pretrained(self.model)
            except Exception:
                tokenizer = None
        # the decoder owns these weights: the o, gate_up and down originals go once the handle holds packed copies
        decoder = RoundDecoder(self.weights(), self.k, rule, threshold, PREFILL_BUCKETS, block_size=block_size,
                               kv_cache_bytes=kv_cache_bytes, max_model_len=self.max_model_len, tokenizer=tokenizer,
                               release_block_weights=True)
        decoder.prepare()
        return decoder
