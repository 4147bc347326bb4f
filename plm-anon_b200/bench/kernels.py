"""Single-kernel microbenchmarks of libplm_native.so (CUDA-event timing, one CUDA graph of `--iters` launches).

    python plm-anon_b200/bench/kernels.py gemm --n-out 16384 --k 2048 --rows 56 --epi silu
    python plm-anon_b200/bench/kernels.py attention --ctx 1024 --k 7 --heads 16 --head-dim 128 --page 16
    python plm-anon_b200/bench/kernels.py verify --vocab 50257 --aux 1024 --rows 7
    python plm-anon_b200/bench/kernels.py norm --rows 56 --hidden 2048

Prints one JSON line per run: microseconds per launch and the algorithmic bytes per launch over that time. With
``--iters 1 --no-graph`` it issues exactly one launch after ``--warmup`` launches, the shape a profiler capture of one
kernel wants.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def _time(fn, iters: int, warmup: int, graph: bool, flush: bool = False) -> float:
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if flush:  # every launch timed alone after 256 MB of writes have evicted L2 (weights and KV come from HBM)
        buf = torch.empty(64 * 2**20, dtype=torch.float32, device="cuda")
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for start, end in events:
            buf.add_(1.0)
            start.record()
            fn()
            end.record()
        torch.cuda.synchronize()
        return 1000 * sum(start.elapsed_time(end) for start, end in events) / iters
    if graph:
        g = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.current_stream().wait_stream(stream)
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
    else:
        def run():
            for _ in range(iters):
                fn()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    run()
    end.record()
    torch.cuda.synchronize()
    return 1000 * start.elapsed_time(end) / iters


def bench_gemm(args, ctx):
    import torch

    from plm import native

    w = (torch.randn(args.n_out, args.k, device="cuda") * 0.02).bfloat16()
    x = torch.randn(256, args.k, device="cuda").bfloat16()
    out = torch.empty(256, args.n_out, device="cuda", dtype=torch.bfloat16)
    kind = {"store": native.EPI_STORE, "silu": native.EPI_SILU_MUL}[args.epi]
    epi = native.GemmEpilogue(kind=kind, gate_offset=args.n_out // 2)
    fn = lambda: native.gemm(ctx, w, x, args.rows, out=out, epi=epi, splits=args.splits)  # noqa: E731
    us = _time(fn, args.iters, args.warmup, not args.no_graph, args.flush)
    ctx.check()
    nbytes = args.n_out * args.k * 2 + args.rows * args.k * 2 + args.rows * args.n_out * 2
    return {"kernel": "skinny_gemm_kernel", "n_out": args.n_out, "k": args.k, "rows": args.rows, "epi": args.epi,
            "us": us, "GB/s": nbytes / us / 1e3, "bytes": nbytes}


def bench_attention(args, ctx):
    import torch

    from plm import native

    k, page, heads, hd = args.k_round, args.page, args.heads, args.head_dim
    rows = k + k * k
    from plm.mask import round_layout

    _, _, depth, own = round_layout([k] * k)
    total = args.ctx + rows
    max_pages = -(-total // page)
    num_pages = 2 * max_pages
    table = torch.randperm(num_pages, device="cuda")[:max_pages].to(torch.int32)
    kc = torch.randn(num_pages, heads, page, hd, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    q = torch.randn(rows, heads, hd, device="cuda").bfloat16()
    out = torch.empty(rows, heads * hd, device="cuda", dtype=torch.bfloat16)
    offset = torch.tensor([args.ctx], dtype=torch.int64, device="cuda")
    d32, o32 = depth.to(torch.int32).cuda(), own.to(torch.int32).cuda()
    desc = native.AttentionDesc(dtype=native.PLM_BF16, q=q.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
                                block_table=table.data_ptr(), max_pages=max_pages, num_pages=num_pages,
                                page_size=page, offset=offset.data_ptr(), rows=rows, depth=d32.data_ptr(),
                                own_start=o32.data_ptr(), num_heads=heads, num_kv_heads=heads, head_dim=hd,
                                out=out.data_ptr(), splits=args.splits, max_keys=total)
    fn = lambda: native.attention(ctx, desc)  # noqa: E731
    us = _time(fn, args.iters, args.warmup, not args.no_graph, args.flush)
    ctx.check()
    nbytes = total * heads * hd * 2 * 2 + 2 * rows * heads * hd * 2
    return {"kernel": "round_attention_kernel", "ctx": args.ctx, "rows": rows, "heads": heads, "head_dim": hd,
            "page": page, "us": us, "GB/s": nbytes / us / 1e3, "bytes": nbytes}


def bench_norm(args, ctx):
    import torch

    from plm import native

    x = torch.randn(args.rows, args.hidden, device="cuda").bfloat16()
    res = torch.randn(args.rows, args.hidden, device="cuda").bfloat16()
    w = torch.ones(args.hidden, device="cuda").bfloat16()
    normed = torch.empty_like(x)
    desc = native.AddRmsNormDesc(dtype=native.PLM_BF16, x=x.data_ptr(), residual=res.data_ptr(),
                                 normed=normed.data_ptr(), weight=w.data_ptr(), rows=args.rows, hidden=args.hidden,
                                 eps=1e-5, gather_row=-1, gathered=None)
    fn = lambda: native.add_rmsnorm(ctx, desc)  # noqa: E731
    us = _time(fn, args.iters, args.warmup, not args.no_graph, args.flush)
    ctx.check()
    nbytes = args.rows * args.hidden * 2 * 4 + args.hidden * 2  # read x, residual; write residual, normed; weight
    return {"kernel": "add_norm_kernel", "rows": args.rows, "hidden": args.hidden, "us": us, "GB/s": nbytes / us / 1e3,
            "bytes": nbytes}


def bench_verify(args, ctx):
    import torch

    from plm import native

    logits = (torch.randn(args.rows, args.vocab, device="cuda") * 2).bfloat16().float()
    table = (torch.randn(args.vocab, args.aux, device="cuda") * 0.3).bfloat16()
    aux_buf = torch.randint(0, args.aux, (8192,), device="cuda")
    verify = torch.zeros(args.rows, dtype=torch.int64, device="cuda")
    flags = torch.zeros(args.rows, dtype=torch.int32, device="cuda")
    desc = native.VerifyDesc(dtype=native.PLM_BF16, logits=logits.data_ptr(), n_rows=args.rows, vocab=args.vocab,
                             logits_stride=args.vocab, table=table.data_ptr(), aux=args.aux,
                             aux_buf=aux_buf.data_ptr(), aux_len=8192, top_m=128, shortlist=8, rounds=2, sweeps=12,
                             epsilon=0.15, refocus=0.35, endpoint=0.0087, verify=verify.data_ptr(),
                             flags=flags.data_ptr(), threshold=-1.0, book=native.Bookkeeping(mode=0))
    phases = torch.zeros(args.rows, 16, dtype=torch.int64, device="cuda")
    desc.dbg_phase_ns = phases.data_ptr()
    fn = lambda: native.verify_decode(ctx, desc)  # noqa: E731
    us = _time(fn, args.iters, args.warmup, not args.no_graph, args.flush)
    ctx.check()
    names = ["stats", "rule", "slice_select", "merge_copy", "merge_sort", "staging", "quota_spread_prior", "condense0",
             "fit0", "condense1", "fit1", "final_sync", "argmin"]
    nbytes = args.rows * (args.vocab * 4 + 2 * 128 * args.aux * 2)
    return {"kernel": "verify_decode_kernel", "rows": args.rows, "vocab": args.vocab, "aux": args.aux, "us": us,
            "GB/s": nbytes / us / 1e3, "bytes": nbytes,
            "phase_end_us": dict(zip(names, (phases[0].float() / 1000).tolist()))}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = parser.add_subparsers(dest="kernel", required=True)
    for name in ("gemm", "attention", "verify", "norm"):
        p = sub.add_parser(name)
        p.add_argument("--iters", type=int, default=20)
        p.add_argument("--warmup", type=int, default=3)
        p.add_argument("--no-graph", action="store_true")
        p.add_argument("--flush", action="store_true", help="evict L2 before every timed launch")
        p.add_argument("--splits", type=int, default=0)
        if name == "gemm":
            p.add_argument("--n-out", type=int, default=16384)
            p.add_argument("--k", type=int, default=2048)
            p.add_argument("--rows", type=int, default=56)
            p.add_argument("--epi", default="store", choices=("store", "silu"))
        elif name == "attention":
            p.add_argument("--ctx", type=int, default=1024)
            p.add_argument("--k", dest="k_round", type=int, default=7)
            p.add_argument("--heads", type=int, default=16)
            p.add_argument("--head-dim", type=int, default=128)
            p.add_argument("--page", type=int, default=16)
        elif name == "norm":
            p.add_argument("--rows", type=int, default=56)
            p.add_argument("--hidden", type=int, default=2048)
        else:
            p.add_argument("--vocab", type=int, default=50257)
            p.add_argument("--aux", type=int, default=1024)
            p.add_argument("--rows", type=int, default=7)
    args = parser.parse_args()
    from plm import native

    ctx = native.Context()
    fn = {"gemm": bench_gemm, "attention": bench_attention, "verify": bench_verify, "norm": bench_norm}[args.kernel]
    print(json.dumps(fn(args, ctx)))


if __name__ == "__main__":
    main()
