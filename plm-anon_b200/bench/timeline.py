"""In-graph kernel timeline of the round (CUPTI through torch.profiler): where a round's time goes on the device.

    python plm-anon_b200/bench/timeline.py --ctx 1024
    python plm-anon_b200/bench/timeline.py --ctx 4096 --json out.json

Builds the configs[1] workload (random PLM-1.3B-shaped weights, a shuffled 16-token page pool, N(0, 1) K/V, a steady
round at offset ``--ctx``), replays the round's CUDA graph, traces ``--rounds`` replays and reports one of them.
With programmatic dependent launch a kernel starts while its predecessor still runs, so launch durations overlap;
the critical-path share of a launch is the time from the previous launch's end to its own end, and those shares add
up to the round's span.
"""

from __future__ import annotations

import argparse
import collections
import json
import sys
import tempfile
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

KINDS = ("mlp_block", "round_attention", "add_norm", "embed_norm", "verify_decode", "icdf_decode", "commit_kernel",
         "skinny")


def _kind(name: str) -> str:
    return next((k for k in KINDS if k in name), name.split("(")[0][-40:])


def build(shape: str, k: int, page: int, ctx: int, seed: int = 0):
    import torch

    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    cfg = shape_config(shape)
    weights = PLMWeights.random(cfg, seed=seed)
    width = k + k * k
    max_model_len = max(2048, ctx + 1024)
    max_pages = -(-(max_model_len + 2 * width + page) // page)
    num_pages = 2 * max_pages
    page_bytes = cfg.num_layers * 2 * cfg.num_kv_heads * page * cfg.head_dim * 2
    table = torch.randperm(num_pages, generator=torch.Generator().manual_seed(seed))[:max_pages].tolist()
    decoder = RoundDecoder(weights, k, "nucleus", None, block_size=page, kv_cache_bytes=num_pages * page_bytes,
                           max_model_len=max_model_len, block_table=table)
    decoder.prepare()
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    kv = decoder.kv_cache
    for layer in range(kv.shape[0]):
        kv[layer].copy_(torch.randn(kv[layer].shape, generator=g, device="cuda").to(kv.dtype))
    decoder.handle.set_stop(1 << 62)
    decoder.offset_t.fill_(ctx)
    decoder.base_t.fill_(2)
    decoder.out.fill_(-1)
    decoder.anchor.fill_(17)
    decoder.pending.copy_(torch.randint(0, cfg.vocab, (k - 1,), generator=g, device="cuda"))
    decoder._fill_aux(0)
    torch.cuda.synchronize()
    return cfg, decoder


def trace(decoder, rounds: int, warmup: int = 5) -> list[dict]:
    import torch
    from torch.profiler import ProfilerActivity, profile

    for _ in range(warmup):
        decoder.graph.replay()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(rounds):
            decoder.graph.replay()
        torch.cuda.synchronize()
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "trace.json"
        prof.export_chrome_trace(str(path))
        events = [e for e in json.loads(path.read_text())["traceEvents"] if e.get("cat") == "kernel"]
    events.sort(key=lambda e: e["ts"])
    return events


def summarise(events: list[dict], rounds: int) -> dict:
    per_round = len(events) // rounds
    last = events[-per_round:]
    t0 = last[0]["ts"]
    prev_end = t0
    last_gemm = max(i for i, e in enumerate(last) if "skinny" in e["name"])
    launches, kinds = [], collections.OrderedDict()
    for i, e in enumerate(last):
        kind, start, dur = _kind(e["name"]), e["ts"] - t0, e["dur"]
        end = start + dur
        critical = end - (prev_end - t0)
        if kind == "skinny":  # the qkv projections, then lm_head (the round's last GEMM)
            kind = "skinny_gemm (lm_head)" if i == last_gemm else "skinny_gemm (qkv)"
        launches.append({"kernel": kind, "start_us": round(start, 2), "dur_us": round(dur, 2),
                         "critical_us": round(critical, 2)})
        k = kinds.setdefault(kind, {"launches": 0, "dur_us": 0.0, "critical_us": 0.0})
        k["launches"] += 1
        k["dur_us"] += dur
        k["critical_us"] += critical
        prev_end = max(prev_end, e["ts"] + dur)
    span = prev_end - t0
    return {"span_us": round(span, 1), "launches": len(last),
            "kinds": {k: {"launches": v["launches"], "avg_dur_us": round(v["dur_us"] / v["launches"], 2),
                          "critical_us": round(v["critical_us"], 1),
                          "critical_share": round(v["critical_us"] / span, 3)} for k, v in kinds.items()},
            "timeline": launches}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--shape", default="plm-1.3b")
    parser.add_argument("--k", type=int, default=7)
    parser.add_argument("--page", type=int, default=16)
    parser.add_argument("--ctx", type=int, default=1024)
    parser.add_argument("--rounds", type=int, default=3)
    parser.add_argument("--json", default=None, help="write the full per-launch timeline here")
    args = parser.parse_args()
    _, decoder = build(args.shape, args.k, args.page, args.ctx)
    result = summarise(trace(decoder, args.rounds), args.rounds)
    result.update({"shape": args.shape, "k": args.k, "ctx": args.ctx, "page": args.page})
    if args.json:
        Path(args.json).write_text(json.dumps(result, indent=1))
    print(f"round span {result['span_us']} us, {result['launches']} launches (ctx {args.ctx})")
    print("| kernel | launches | avg launch duration us | critical path us | share |")
    print("|---|---|---|---|---|")
    for k, v in result["kinds"].items():
        print(f"| {k} | {v['launches']} | {v['avg_dur_us']} | {v['critical_us']} | {100 * v['critical_share']:.1f}% |")
    layer = [x for x in result["timeline"][1:5]]
    print("one layer (start, duration, critical path; us from the round's start):")
    for x in layer:
        print(f"  {x['kernel']:24s} start {x['start_us']:8.2f}  dur {x['dur_us']:6.2f}  critical {x['critical_us']:6.2f}")


if __name__ == "__main__":
    main()
