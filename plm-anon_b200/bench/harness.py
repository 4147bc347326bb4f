"""Dataset loading, per-prompt speed records and seeded passes (same interface as the reference's bench/harness.py).

A dataset is a JSON list of prompts: strings (tokenised by the model's tokenizer) or lists of token ids. With no
tokenizer and no dataset files on the machine, ``random:<count>:<length>[:<seed>]`` stands for ``count`` prompts of
``length`` token ids uniform in the vocabulary, drawn from a CPU generator seeded with ``seed`` (default 0).
"""

from __future__ import annotations

import argparse
import json
from collections.abc import Callable
from dataclasses import dataclass
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
    """The run flags of the reference's harness (bench/harness.py:42-49): same names, defaults and meaning."""
    parser.add_argument("--max-model-len", type=int, default=4096,
                        help="longest request the decoder is sized for (prompt and continuation together)")
    parser.add_argument("--dataset", required=True,
                        help="a JSON file listing prompts (text or token-id lists), or random:<count>:<length>[:<seed>]")
    parser.add_argument("--prompts", type=int, default=None, help="keep only this many prompts from the start")
    parser.add_argument("--tokens", type=int, default=128,
                        help="continuation length per prompt; with --stop-at-eos, the most it may reach")
    parser.add_argument("--stop-at-eos", action="store_true", help="cut a continuation at its end-of-text token")
    parser.add_argument("--seeds", type=int, nargs="+", default=[0, 1, 2],
                        help="the recorded passes, one per seed; an unrecorded warm-up pass uses the first")
    parser.add_argument("--out", default="results.json", help="where the results file goes")


@dataclass
class Passes:
    """Runs ``generate_one(prompt, seed) -> speed record`` over the whole dataset, once per call of ``run``."""

    generate_one: Callable
    dataset: list

    def run(self, seed: int, label: str) -> list[dict]:
        records = []
        for index, prompt in enumerate(self.dataset):
            record = self.generate_one(prompt, seed)
            records.append(record)
            print(f"{label}: prompt {index + 1}/{len(self.dataset)}, {record['tokens']} tokens, "
                  f"{record['tokens_per_call']:.2f} per round, {record['tokens_per_second']:.1f} tokens/s")
        return records


def _summary_line(summary: dict) -> str:
    return ", ".join(f"{key} {value:.3f}" if isinstance(value, float) else f"{key} {value}"
                     for key, value in summary.items())


def run_passes(described: dict, generate_one: Callable, dataset: list, args: argparse.Namespace) -> dict:
    """The measurement the reference's run_passes makes (bench/harness.py:52-66): the warm-up pass pays graph
    capture and cold clocks and is not recorded; each seed's pass is recorded with its aggregate. The results file
    keeps the reference's layout: {"config": ..., "passes": [{"seed", "aggregate", "results"}]}."""
    passes = Passes(generate_one, dataset)
    passes.run(args.seeds[0], "warm-up (not recorded)")
    recorded = []
    for seed in args.seeds:
        records = passes.run(seed, f"seed {seed}")
        summary = aggregate(records)
        print(f"seed {seed} aggregate: {_summary_line(summary)}")
        recorded.append({"seed": seed, "aggregate": summary, "results": records})
    run = {"seeds": args.seeds, "prompts": len(dataset), "tokens": args.tokens, "stop_at_eos": args.stop_at_eos,
           "max_model_len": args.max_model_len, "dataset": args.dataset}
    result = {"config": {**described, **run}, "passes": recorded}
    Path(args.out).write_text(json.dumps(result, indent=1))
    print(f"results written to {args.out}")
    return result
