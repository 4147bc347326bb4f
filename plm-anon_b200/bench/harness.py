"""Dataset loading, per-prompt speed records and seeded passes (same interface as the reference's bench/harness.py).

A dataset is a JSON list of prompts: strings (tokenised by the model's tokenizer) or lists of token ids. With no
tokenizer and no dataset files on the machine, ``random:<count>:<length>[:<seed>]`` stands for ``count`` prompts of
``length`` token ids uniform in the vocabulary, drawn from a CPU generator seeded with ``seed`` (default 0).
"""

from __future__ import annotations

import argparse
import json
from collections.abc import Callable
from pathlib import Path

import torch


def load_dataset(path: str, count: int | None, vocab: int = 50257) -> list:
    """bench/harness.py:12-16: a JSON list of prompts, optionally only the first ``count``."""
    if path.startswith("random:"):
        parts = path.split(":")
        n, length = int(parts[1]), int(parts[2])
        seed = int(parts[3]) if len(parts) > 3 else 0
        generator = torch.Generator().manual_seed(seed)
        loaded = [torch.randint(vocab, (length,), generator=generator).tolist() for _ in range(n)]
    else:
        loaded = json.loads(Path(path).read_text())
        if not isinstance(loaded, list) or not all(
                isinstance(p, str) or (isinstance(p, list) and all(isinstance(t, int) for t in p)) for p in loaded):
            raise SystemExit(f"{path}: expected a JSON list of prompt strings or token-id lists")
    return loaded if count is None else loaded[:count]


def speed_record(prompt, continuation: str, accepted: list[int], calls: int, tokens: int, ms: float, steady_ms: float,
                 steady_tokens: int) -> dict:
    """bench/harness.py:19-22."""
    return {"prompt": prompt, "continuation": continuation, "accepted_per_call": accepted, "calls": calls,
            "tokens": tokens, "ms": ms, "ms_per_call": steady_ms / calls if calls else 0.0,
            "tokens_per_call": steady_tokens / calls if calls else 0.0,
            "tokens_per_second": tokens / (ms / 1000) if ms else 0.0}


def measure(generate_one: Callable, dataset: list, seed: int) -> list[dict]:
    records = []
    for index, prompt in enumerate(dataset, 1):
        records.append(generate_one(prompt, seed))
        print(f"  [seed {seed}  {index}/{len(dataset)}] {records[-1]['tokens_per_call']:.2f} tok/call  "
              f"{records[-1]['tokens_per_second']:.0f} tok/s")
    return records


def aggregate(records: list[dict]) -> dict:
    """bench/harness.py:33-39: per-pass totals; rates over the steady rounds' time, and end to end over the wall time
    of the whole requests."""
    calls = sum(r["calls"] for r in records)
    tokens = sum(r["tokens"] for r in records)
    steady_ms = sum(r["ms_per_call"] * r["calls"] for r in records)
    wall_ms = sum(r["ms"] for r in records)
    return {"prompts": len(records), "calls": calls, "tokens": tokens,
            "ms_per_call": steady_ms / calls if calls else 0.0,
            "tokens_per_call": tokens / calls if calls else 0.0,
            "tokens_per_second": 1000 * tokens / steady_ms if steady_ms else 0.0,
            "e2e_tokens_per_second": 1000 * tokens / wall_ms if wall_ms else 0.0}


def add_run_arguments(parser: argparse.ArgumentParser) -> None:
    """bench/harness.py:42-49."""
    parser.add_argument("--max-model-len", type=int, default=4096, help="prompt plus generated tokens")
    parser.add_argument("--dataset", required=True,
                        help="JSON list of prompt strings or token-id lists, or random:<count>:<length>[:<seed>]")
    parser.add_argument("--prompts", type=int, default=None, help="use only the first N prompts")
    parser.add_argument("--tokens", type=int, default=128, help="generated tokens per prompt (a ceiling with --stop-at-eos)")
    parser.add_argument("--stop-at-eos", action="store_true", help="end each continuation at the end-of-text token")
    parser.add_argument("--seeds", type=int, nargs="+", default=[0, 1, 2],
                        help="one measured pass per seed, after a discarded warm-up pass")
    parser.add_argument("--out", default="results.json")


def run_passes(described: dict, generate_one: Callable, dataset: list, args: argparse.Namespace) -> dict:
    """bench/harness.py:52-66: a discarded warm-up pass, then one measured pass per seed, written as one file."""
    print("=== warm-up pass (discarded)")
    measure(generate_one, dataset, args.seeds[0])
    passes = []
    for seed in args.seeds:
        print(f"=== seed {seed}")
        records = measure(generate_one, dataset, seed)
        passes.append({"seed": seed, "aggregate": aggregate(records), "results": records})
        print("  " + "  ".join(f"{key}={value:.3f}" if isinstance(value, float) else f"{key}={value}"
                               for key, value in passes[-1]["aggregate"].items()))
    described = dict(described) | {"seeds": args.seeds, "prompts": len(dataset), "tokens": args.tokens,
                                   "stop_at_eos": args.stop_at_eos, "max_model_len": args.max_model_len,
                                   "dataset": args.dataset}
    result = {"config": described, "passes": passes}
    Path(args.out).write_text(json.dumps(result, indent=1))
    print(f"  -> {args.out}")
    return result
