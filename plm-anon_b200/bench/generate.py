"""Generate a continuation for every prompt in a dataset, once per seed, and write a results file with per-prompt
speed, on the native round engine (same flags and results file as the reference's bench/generate.py).

    python -m bench.generate --model synthetic:plm-1.3b --match exact --k 7 \\
        --dataset random:4:256 --tokens 512 --seeds 0 1 2 --out results.json

One process runs the whole dataset ``1 + len(--seeds)`` times: a discarded warm-up pass, which pays graph capture and
a cold clock, then one pass per seed. The seed drives the request's auxiliary cell stream. ``--model`` is an export
directory (config.json + safetensors with the auxiliary scheme) or ``synthetic:<shape>[:seed=<n>]``.

``--ar --ar-sampler voronoi`` is the AR-Voronoi comparator (plm/voronoi_ar.py, bench/ar.py): one verify row per step,
which is a round with k = 1 on the same engine, and decodes the same tokens as ``--match exact``. The other AR
samplers and the EAGLE-3 / Fast-dLLM v2 comparators (``--eagle3``, ``--fdv2``) run stock vLLM or third-party packages
in the reference and exit with a message.
"""

from __future__ import annotations

import argparse
import time
from collections.abc import Callable

from .harness import add_run_arguments, load_dataset, run_passes, speed_record
from plm.rounds import SETTINGS, RoundConfig

KV_BLOCK_SIZE = 64        # bench/engine.py:4
KV_CACHE_BYTES = 1 << 30  # bench/engine.py:5


def add_arguments(parser: argparse.ArgumentParser) -> None:
    """bench/generate.py:25-40."""
    parser.add_argument("--model", required=True, help="an export directory, or synthetic:<shape>[:seed=<n>]")
    parser.add_argument("--setting", default="posttrain", choices=tuple(SETTINGS),
                        help="posttrain: k 7 (exact) / 10 (relaxed), nucleus 0.94. pretrain: k 6, probability floor 2e-3")
    parser.add_argument("--mode", default="fast", choices=("fast", "default"),
                        help="accepted for compatibility: both run the native sm_100a kernels")
    parser.add_argument("--match", default="exact", choices=("exact", "relaxed"),
                        help="exact, or relaxed (the setting's looser accept rule)")
    parser.add_argument("--k", type=int, help="proposal length per round; default from --setting")
    parser.add_argument("--block-size", type=int, default=KV_BLOCK_SIZE, help="KV page size in tokens")
    parser.add_argument("--dtype", default="", choices=("", "bfloat16", "float16"),
                        help="weights' dtype on the GPU; default: the export's own (the kernels run bfloat16 and "
                             "float16; naming the other converts the weights)")
    parser.add_argument("--ar", action="store_true", help="autoregressive decoding: one Voronoi-decoded row per step")
    parser.add_argument("--ar-sampler", default="voronoi", choices=("voronoi", "icdf", "topk", "greedy"),
                        help="voronoi: the PLM's own decode rule on the seeded cells, token-identical to --match exact "
                             "(the only sampler built on this engine)")
    parser.add_argument("--eagle3", default="", help="EAGLE-3 head (not built on this engine)")
    parser.add_argument("--fdv2", action="store_true", help="Fast-dLLM v2 (not built on this engine)")


def run_plm(decoder, prompt, tokens: int, stop_at_eos: bool, seed: int) -> dict:
    """bench/generate.py:43-52: one request, its accepted count per round from the decoder's round record."""
    started = time.perf_counter()
    first_round = int(decoder.sequence_step.item())
    result = decoder.generate(prompt, tokens, seed=seed, stop_at_eos=stop_at_eos)
    accepted = decoder.round_sequence[first_round:int(decoder.sequence_step.item())].tolist()
    ms = 1000 * (time.perf_counter() - started)
    record = speed_record(prompt if isinstance(prompt, str) else len(prompt), result.text, accepted,
                          result.steady_rounds, len(result.token_ids), ms, result.steady_ms, result.steady_tokens)
    record["tokens_per_second"] = result.tokens_per_second
    record["token_ids"] = result.token_ids
    return record


def round_config(args: argparse.Namespace) -> RoundConfig:
    """The RoundConfig the flags select (bench/generate.py:67-71). AR-Voronoi is exact matching with k = 1."""
    if args.ar:
        return RoundConfig(model=args.model, setting=args.setting, mode=args.mode, match="exact", k=1,
                           dtype=args.dtype or None, max_model_len=args.max_model_len)
    return RoundConfig(model=args.model, setting=args.setting, mode=args.mode, match=args.match, k=args.k,
                       dtype=args.dtype or None, max_model_len=args.max_model_len)


def plm_generator(args: argparse.Namespace) -> tuple[dict, Callable]:
    """bench/generate.py:67-71 (and the AR-Voronoi comparator of 55-64 as a k = 1 round)."""
    round_config_ = round_config(args)
    decoder = round_config_.build(kv_cache_bytes=KV_CACHE_BYTES, block_size=args.block_size)
    decoding = "ar-voronoi" if args.ar else round_config_.match
    described = {"decoding": decoding, **round_config_.describe()}
    return described, lambda prompt, seed: run_plm(decoder, prompt, args.tokens, args.stop_at_eos, seed)


def build_generator(args: argparse.Namespace) -> tuple[dict, Callable]:
    if args.eagle3 or args.fdv2:
        raise SystemExit("--eagle3 and --fdv2 are not built on this engine: it runs PLM parallel rounds")
    if args.ar and args.ar_sampler != "voronoi":
        raise SystemExit(f"--ar-sampler {args.ar_sampler} is not built on this engine (voronoi is: a k = 1 round)")
    return plm_generator(args)


def main(argv: list[str] | None = None) -> dict:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_arguments(parser)
    add_run_arguments(parser)
    args = parser.parse_args(argv)
    described, generate_one = build_generator(args)
    vocab = 50257
    if args.model.startswith("synthetic:"):
        from plm.model import shape_config

        vocab = shape_config(args.model.split(":")[1]).vocab
    dataset = load_dataset(args.dataset, args.prompts, vocab)
    return run_passes(described, generate_one, dataset, args)


if __name__ == "__main__":
    main()
