"""Benchmark of the PLM round step on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

Workload (the single-round microbenchmark): PLM-1.3B shape (24 layers, d 2048, 16x128
MHA, SiLU-gated MLP 8192, vocab 50257), bf16 N(0, 0.02) weights from seed 0, k = 7 (7 verify + 49 proposal rows),
exact match with Voronoi sampling, KV context of 1024 tokens in 16-token pages through a shuffled block table, K/V
~ N(0, 1). A step is one steady round (a replay of the captured round graph); the state carries over between
steps, so the context grows by the accepted tokens. Weights (3.4 GB) exceed L2, so no flush is needed.

  value   accepted tokens/s over all GPUs, device-timed with CUDA events (inputs resident in HBM).
  e2e     the same metric through the public API: RoundDecoder.generate on BASELINE configs[2]'s requests (a
          256-token prompt copied from pinned host memory, 512 new tokens, seeds 0, 1, 2 in turn), the rounds kept in
          flight by the device-side stop, the tokens read back; --e2e-requests per rank.
  roofline  the dominant kernel (the layer blocks of a round: o, its norm, gate_up and down of every layer, launched
          exactly as in the round) timed live by CUDA events: weight bytes / time, against the measured HBM copy
          bandwidth.
  round_roofline  all algorithmic bytes of a round (weights, KV read and written, Voronoi gathers) / round time.
  cpu_baseline    the CPU oracle's round (oracle/model.py, torch on all host threads) on a bounded sample.

Multi-GPU (torchrun, one process per GPU): replicas only — every rank runs the same workload on its own GPU
(weak scaling), no data-path collective; the elapsed time is the maximum over ranks.
``--impl reference`` times the reference arm: the CPU round oracle (the reference's path has no CPU implementation of
its own), built from seeded CPU generators and run on all host cores for the same steps, rank 0 only; it loads no
GPU library of this repository.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "plm-anon_b200"), str(ROOT)]

METRIC = "accepted tokens/sec/GPU at batch 1 (PLM-1.3B shape, k=7); round latency µs; %HBM"
UNIT = "tokens/s"
SHAPE, K, PAGE, CTX = "plm-1.3b", 7, 16, 1024
PROMPT_E2E, TOKENS_E2E = 256, 512


def _peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.device_index, self.samples, self.proc = device_index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device_index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            deadline = time.perf_counter() + 3.0  # the timed region starts once sampling runs
            while not self.samples and time.perf_counter() < deadline:
                time.sleep(0.01)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.samples[0][2]) if self.samples[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(self.samples)}


def round_bytes(cfg, ctx: float, k: int) -> dict:
    """Algorithmic HBM bytes of one round (the per-round figure of the roofline)."""
    b = 2
    hd, kvh, L = cfg.head_dim, cfg.num_kv_heads, cfg.num_layers
    q_size, kv_size = cfg.num_heads * hd, kvh * hd
    per_layer = ((q_size + 2 * kv_size) * cfg.hidden + cfg.hidden * q_size + 2 * cfg.intermediate * cfg.hidden
                 + cfg.hidden * cfg.intermediate) * b
    weights = L * per_layer + cfg.vocab * cfg.hidden * b
    w = k + k * k
    kv_read = ctx * L * 2 * kv_size * b
    kv_write = w * L * 2 * kv_size * b
    embed = w * cfg.hidden * b
    voronoi = k * (2 * cfg.top_m * cfg.aux_vocab * b + cfg.top_m * 64 * b)
    logits = 2 * k * cfg.vocab * 4
    return {"weights": weights, "kv_read": kv_read, "kv_write": kv_write, "embed": embed, "voronoi": voronoi,
            "logits": logits, "total": weights + kv_read + kv_write + embed + voronoi + logits}


def reduce_over_ranks(dist, elapsed_ms: float, tokens: float, device: str = "cuda") -> tuple[float, float]:
    """Replicas only: the job's time is the slowest rank's, its tokens the sum over ranks."""
    import torch

    if dist is None:
        return float(elapsed_ms), float(tokens)
    mx = torch.tensor([float(elapsed_ms)], dtype=torch.float64, device=device)
    sm = torch.tensor([float(tokens)], dtype=torch.float64, device=device)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx[0]), float(sm[0])


def _dist():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        return rank, world, local, dist
    if torch.cuda.is_available():
        torch.cuda.set_device(0)
    return 0, 1, 0, None


def _setup_decoder(seed: int = 0, separate_mlp: bool = False, ctx: int = CTX):
    """The configs[1] workload: weights, a decoder over a shuffled pool, a ``ctx``-token N(0, 1) context."""
    import torch

    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    cfg = shape_config(SHAPE)
    weights = PLMWeights.random(cfg, seed=seed)
    max_model_len = max(2048, ctx + 1024)
    max_pages = -(-(max_model_len + 2 * (K + K * K) + PAGE) // PAGE)
    num_pages = 2 * max_pages
    page_bytes = cfg.num_layers * 2 * cfg.num_kv_heads * PAGE * cfg.head_dim * 2
    g = torch.Generator().manual_seed(seed)
    table = torch.randperm(num_pages, generator=g)[:max_pages].tolist()
    decoder = RoundDecoder(weights, K, "nucleus", None, block_size=PAGE, kv_cache_bytes=num_pages * page_bytes,
                           max_model_len=max_model_len, block_table=table, separate_mlp=separate_mlp)
    decoder.prepare()
    return cfg, weights, decoder


def _seed_context(decoder, cfg, seed: int = 1, ctx: int = CTX) -> None:
    """K/V ~ N(0, 1) bf16 over the pool, then the request state of a steady round at offset ``ctx`` (no stop)."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    kv = decoder.kv_cache
    for layer in range(kv.shape[0]):
        kv[layer].copy_(torch.randn(kv[layer].shape, generator=g, device="cuda", dtype=torch.float32).bfloat16())
    decoder.handle.set_stop(1 << 62)
    decoder.offset_t.fill_(ctx)
    decoder.base_t.fill_(2)
    decoder.out.fill_(-1)
    decoder.anchor.fill_(17)
    decoder.pending.copy_(torch.randint(0, cfg.vocab, (K - 1,), generator=g, device="cuda"))
    decoder._fill_aux(0)
    torch.cuda.synchronize()


def _gemm_graph(decoder, cfg):
    """A graph of exactly the round's weight GEMM launches (same weights, buffers, epilogues and splits)."""
    import torch

    from plm import native

    h, w, c = decoder, decoder.weights, cfg
    ctx = native.Context()
    rows = decoder.width
    x = torch.zeros(256, c.hidden, dtype=torch.bfloat16, device="cuda")
    xi = torch.zeros(256, c.intermediate, dtype=torch.bfloat16, device="cuda")
    xa = torch.zeros(256, c.num_heads * c.head_dim, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(256, max(c.hidden, c.intermediate), dtype=torch.bfloat16, device="cuda")
    q = torch.zeros(256, c.num_heads * c.head_dim, dtype=torch.bfloat16, device="cuda")
    positions = torch.arange(rows, dtype=torch.int32, device="cuda") + CTX
    slots = torch.arange(rows, dtype=torch.int64, device="cuda") + CTX
    tiles = native.gemm_tiles(native.EPI_LOGITS, c.vocab)
    logits = torch.zeros(K, c.vocab, dtype=torch.float32, device="cuda")
    best_val = torch.zeros(tiles, rows, dtype=torch.float32, device="cuda")
    best_idx = torch.zeros(tiles, rows, dtype=torch.int32, device="cuda")
    kv = h.kv_cache

    def body():
        for layer in range(c.num_layers):
            e = native.GemmEpilogue(kind=native.EPI_QKV_ROPE, q_out=q.data_ptr(), k_cache=kv[layer, 0].data_ptr(),
                                    v_cache=kv[layer, 1].data_ptr(), positions=positions.data_ptr(),
                                    slots=slots.data_ptr(), cos_sin=h.cos_sin.data_ptr(), num_heads=c.num_heads,
                                    num_kv_heads=c.num_kv_heads, head_dim=c.head_dim, page_size=PAGE,
                                    num_slots=h.num_pages * PAGE, max_pos=h.cos_sin.shape[0])
            native.gemm(ctx, w.qkv[layer], x, rows, epi=e)
            native.gemm(ctx, w.o[layer], xa, rows, out=y[:, : c.hidden])
            native.gemm(ctx, w.gate_up[layer], x, rows, out=y[:, : c.intermediate],
                        epi=native.GemmEpilogue(kind=native.EPI_SILU_MUL, gate_offset=c.intermediate))
            native.gemm(ctx, w.down[layer], xi, rows, out=y[:, : c.hidden])
        native.gemm(ctx, w.lm_head, x, rows,
                    epi=native.GemmEpilogue(kind=native.EPI_LOGITS, verify_logits=logits.data_ptr(),
                                            best_val=best_val.data_ptr(), best_idx=best_idx.data_ptr(), n_verify=K,
                                            vocab=c.vocab))

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        body()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    keep = (ctx, x, xi, xa, y, q, positions, slots, logits, best_val, best_idx)
    return graph, keep, 4 * c.num_layers + 1


def _block_graph(decoder, cfg):
    """A graph of exactly the round's layer-block launches (o projection, its norm, gate_up and down of every layer,
    over the round's rows), each after the counter reset a forward's prologue does."""
    import torch

    body = lambda: [decoder.handle.layer_block(layer, decoder.width) for layer in range(cfg.num_layers)]  # noqa: E731
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        body()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    return graph, (), cfg.num_layers


def block_weight_bytes(cfg) -> int:
    """Weight bytes one round's layer blocks stream: o, gate_up and down of every layer."""
    q_size = cfg.num_heads * cfg.head_dim
    return cfg.num_layers * 2 * (cfg.hidden * q_size + 3 * cfg.intermediate * cfg.hidden)


def _time_graph(graph, reps: int) -> float:
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


def cpu_baseline(weights_gpu, decoder, cfg, rounds: int = 1) -> dict:
    """The CPU oracle's steady round on the same model, context and state (oracle/model.py), all host threads."""
    import numpy as np
    import torch

    from oracle import model as omodel
    from oracle import voronoi as ov

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    shape = omodel.ModelShape(cfg.num_layers, cfg.hidden, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                              cfg.intermediate, cfg.vocab, cfg.aux_vocab, cfg.num_aux_tokens, cfg.rms_eps,
                              cfg.rope_theta, decoder.cos_sin.shape[0])
    named = {key: ([t.cpu() for t in v] if isinstance(v, list) else v.cpu()) for key, v in weights_gpu.named().items()}
    table = decoder.handle.state()
    block_table = torch.from_numpy(np.asarray(
        __import__("plm.native", fromlist=["device_view"]).device_view(table.block_table, (decoder.max_pages,),
                                                                       torch.int32).cpu().numpy()))
    om = omodel.OracleModel(shape, named, "bfloat16", PAGE, decoder.num_pages, block_table.numpy(),
                            cos_sin=decoder.cos_sin.cpu())
    om.kv.copy_(decoder.kv_cache.float().cpu())
    oracle = omodel.RoundOracle(om, decoder.table.float().cpu().numpy(), K, "nucleus", None,
                                ov.VoronoiConfig(cfg.top_m, cfg.shortlist, cfg.rounds, cfg.sweeps),
                                capacity=decoder.out.numel(), aux_stream=decoder.aux_buf.cpu().numpy())
    st = oracle.state
    st.offset, st.base = int(decoder.offset_t), int(decoder.base_t)
    st.anchor, st.pending = int(decoder.anchor[0]), decoder.pending.cpu().numpy().copy()
    tokens = 0
    started = time.perf_counter()
    for _ in range(rounds):
        tokens += oracle.round() + 1
    seconds = time.perf_counter() - started
    return {"value": tokens / seconds, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{rounds} steady round(s) of the configs[1] workload (1.3B shape, k=7, ctx {st.offset}) by the CPU "
                      f"oracle (torch fp32 forward + numpy Voronoi), {seconds:.2f} s",
            "seconds_per_round": seconds / rounds}


def _cpu_workload(seed: int = 0, ctx: int = CTX):
    """The configs[1] workload built on the CPU alone (no GPU, no library of this repository): seeded bf16 weights,
    the Voronoi cost table -(aux_vocab . lm_head^T)^T rounded to bf16, a shuffled block table, K/V ~ N(0, 1) over the
    pool and the state of a steady round at offset ``ctx``, as the CPU round oracle that stands in for the reference's
    round (its own path needs vLLM and a GPU)."""
    import numpy as np
    import torch

    from oracle import model as omodel
    from oracle import voronoi as ov
    from plm.model import PLMWeights, shape_config

    cfg = shape_config(SHAPE)
    weights = PLMWeights.random(cfg, seed=seed, device="cpu")
    max_model_len = max(2048, ctx + 1024)
    max_pages = -(-(max_model_len + 2 * (K + K * K) + PAGE) // PAGE)
    num_pages = 2 * max_pages
    g = torch.Generator().manual_seed(seed)
    block_table = torch.randperm(num_pages, generator=g)[:max_pages].numpy().astype(np.int64)
    cos_sin = omodel.rope_cache(cfg.head_dim, max(cfg.max_pos, max_pages * PAGE), cfg.rope_theta, torch.bfloat16)
    shape = omodel.ModelShape(cfg.num_layers, cfg.hidden, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                              cfg.intermediate, cfg.vocab, cfg.aux_vocab, cfg.num_aux_tokens, cfg.rms_eps,
                              cfg.rope_theta, cos_sin.shape[0])
    model = omodel.OracleModel(shape, weights.named(), "bfloat16", PAGE, num_pages, block_table, cos_sin=cos_sin)
    model.kv.normal_(0.0, 1.0, generator=g)
    model.kv.copy_(model.kv.bfloat16().float())
    scores = weights.aux_vocab.float() @ weights.lm_head.float().T
    table = (-scores.bfloat16().float()).T.contiguous().numpy()
    aux = torch.randint(cfg.aux_vocab, (8192,), generator=torch.Generator().manual_seed(0)).numpy()
    oracle = omodel.RoundOracle(model, table, K, "nucleus", None,
                                ov.VoronoiConfig(cfg.top_m, cfg.shortlist, cfg.rounds, cfg.sweeps),
                                capacity=max_pages * PAGE, aux_stream=aux)
    st = oracle.state
    st.offset, st.base, st.anchor = ctx, 2, 17
    st.pending = torch.randint(0, cfg.vocab, (K - 1,), generator=g).numpy().astype(np.int64)
    del weights
    return cfg, oracle


def workload_config(ctx: int, world: int) -> dict:
    """The ``config`` of both arms' lines (the same workload, whichever arm runs it)."""
    return {"workload": f"BASELINE configs[1]: single-round microbenchmark, PLM-1.3B shape, k=7 (56 rows), exact "
                        f"match + Voronoi, ctx {ctx} (+ accepted tokens), 16-token pages, shuffled block table, "
                        "K/V ~ N(0,1)", "model": SHAPE, "k": K, "rows": K + K * K, "ctx_start": ctx,
            "page_size": PAGE, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (3.4 GB weights per round), no flush"}


def run_reference(args) -> None:
    """Reference arm: the CPU round oracle on all host threads, built and run on the CPU only, for the same steps."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:  # replicas: one host baseline per box
        return
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t_setup = time.perf_counter()
    cfg, oracle = _cpu_workload(ctx=args.ctx)
    setup_s = time.perf_counter() - t_setup
    for _ in range(args.warmup):
        oracle.round()
    base0 = oracle.state.base
    started = time.perf_counter()
    for _ in range(args.steps):
        oracle.round()
    seconds = time.perf_counter() - started
    tokens = oracle.state.base - base0
    value = tokens / seconds
    sample = (f"{args.steps} steady rounds (after {args.warmup} warm-up rounds) of the configs[1] workload by the CPU "
              f"round oracle (torch fp32 forward over bf16 values + numpy Voronoi), {seconds:.2f} s; built on the "
              f"CPU in {setup_s:.1f} s")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * seconds / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": workload_config(args.ctx, 1), "round_us": 1e6 * seconds / args.steps,
            "tokens_per_round": tokens / args.steps,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def write_reference_export(directory: Path, seed: int = 0) -> None:
    """A synthetic PLM-1.3B export both engines load: seeded bf16 weights (lm_head padded to the embedding's rows,
    as a vLLM Llama head expects) and a word-level tokenizer whose token i is the text "w<i>"."""
    import torch
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    from plm.model import PLMWeights, shape_config

    cfg = shape_config(SHAPE)
    w = PLMWeights.random(cfg, seed=seed)
    w.lm_head = torch.cat([w.lm_head, torch.zeros(cfg.vocab_rows - cfg.vocab, cfg.hidden, dtype=w.lm_head.dtype,
                                                  device=w.lm_head.device)])
    w.save_export(directory)
    tok = Tokenizer(models.WordLevel(vocab={f"w{i}": i for i in range(cfg.vocab)}, unk_token="w0"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="w0", eos_token=f"w{cfg.vocab - 1}").save_pretrained(
        directory)


def run_reference_gpu(args) -> None:
    """The reference's own round (baseline/_ref through vLLM, --mode default and fast) and this engine's, on the same
    export, prompt and GPU: one request of a 256-token prompt and 512 new tokens each (after a warm-up request)."""
    import tempfile

    import torch

    if int(os.environ.get("RANK", "0")) != 0:
        return
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "plm").exists():
        print(json.dumps({"impl": "reference-gpu", "unavailable": "the reference is not installed in baseline/_ref"}))
        return
    from plm.rounds import RoundConfig

    seed, tokens = 0, TOKENS_E2E
    with tempfile.TemporaryDirectory() as tmp:
        export = Path(tmp) / "plm-1.3b"
        write_reference_export(export)
        results = {}
        for mode in ("default", "fast"):
            env = dict(os.environ, PYTHONPATH=str(ref))
            proc = subprocess.run([sys.executable, str(ROOT / "plm-anon_b200" / "bench" / "reference_gpu.py"),
                                   str(export), mode, str(seed), str(tokens)], capture_output=True, text=True, env=env,
                                  timeout=1200)
            lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
            errors = [line for line in (proc.stderr + proc.stdout).splitlines()
                      if ("Error" in line or "no tuned tile" in line) and "prime_rl" not in line]
            results[mode] = json.loads(lines[-1]) if proc.returncode == 0 and lines else {
                "failed": (errors or proc.stderr.strip().splitlines() or ["no output"])[-1][:400]}
        decoder = RoundConfig(model=str(export), setting="posttrain", mode="fast", match="exact", k=7,
                              dtype="bfloat16", max_model_len=2048).build(kv_cache_bytes=1 << 30, block_size=16)
        ids = torch.randint(0, shape_config_vocab(), (256,), generator=torch.Generator().manual_seed(seed))
        prompt = " ".join(f"w{int(i)}" for i in ids)
        decoder.generate(prompt, 64, seed=0, stop_at_eos=False)
        res = decoder.generate(prompt, tokens, seed=0, stop_at_eos=False)
        decoder.check()
        ours = {"steady_rounds": res.steady_rounds, "steady_ms": res.steady_ms,
                "round_us": 1000.0 * res.steady_ms / max(res.steady_rounds, 1), "tokens": len(res.token_ids),
                "seconds": res.seconds, "tokens_per_second": len(res.token_ids) / res.seconds}
        decoder.close()
    print(json.dumps({"impl": "reference-gpu", "unit": UNIT, "workload": "PLM-1.3B shape, k=7, exact match + Voronoi, "
                      "256-token prompt, 512 new tokens, 16-token pages, one request after a warm-up request",
                      "reference": results, "native": ours}))


def shape_config_vocab() -> int:
    from plm.model import shape_config

    return shape_config(SHAPE).vocab


# DRAM bytes (read + write) of the weight GEMMs of one round of the benchmark shape, from one ncu capture of each
# GEMM shape at 56 rows: 24 x (qkv 25.47 + o 8.69 + gate_up 68.12 + down 34.64) MB + lm_head 209.7 MB. Used for the
# separate-launch configuration.
GEMM_DRAM_BYTES_PER_ROUND = 3.495e9
# DRAM bytes (read + write) of one layer-block launch of the benchmark shape, from one ncu capture of a block of a
# 2-layer model of the same shape: 134.91 MB read + 4.53 MB written. The reads are the block's own
# 109.7 MB (packed weights and row operands) plus the 25.2 MB of the next layer's qkv weights that its tail
# prefetches into L2, which the qkv GEMM then reads from L2 instead of DRAM.
BLOCK_DRAM_BYTES_PER_LAUNCH = 139.4e6
BLOCK_PREFETCH_BYTES_PER_LAUNCH = 25.2e6


def run_native(args) -> None:
    import torch

    rank, world, local, dist = _dist()
    cfg, weights, decoder = _setup_decoder(separate_mlp=args.separate_mlp, ctx=args.ctx)
    _seed_context(decoder, cfg, ctx=args.ctx)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        decoder.graph.replay()
    torch.cuda.synchronize()
    decoder.check()
    _seed_context(decoder, cfg, ctx=args.ctx)
    base0, ctx0 = int(decoder.base_t), int(decoder.offset_t)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            decoder.graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    decoder.check()
    tokens = int(decoder.base_t) - base0
    ctx_mean = (ctx0 + int(decoder.offset_t)) / 2
    elapsed_ms, total_tokens = reduce_over_ranks(dist, elapsed_ms, tokens)
    ms_per_step = elapsed_ms / args.steps
    value = total_tokens / (elapsed_ms / 1000)

    # dominant kernel, timed live: the layer blocks (o, its norm, gate_up, down of every layer), or with separate
    # launches the round's weight GEMMs
    bytes_ = round_bytes(cfg, ctx_mean, K)
    peak, peak_kind = _peaks()
    if args.separate_mlp:
        graph, keep, dom_launches = _gemm_graph(decoder, cfg)
        dom_kernel, dom_bytes, dom_traffic = "skinny_gemm_kernel (all weight GEMMs of a round)", bytes_["weights"], \
            GEMM_DRAM_BYTES_PER_ROUND
    else:
        graph, keep, dom_launches = _block_graph(decoder, cfg)
        dom_kernel, dom_bytes = "mlp_block_kernel (the layer blocks of a round)", block_weight_bytes(cfg)
        dom_traffic = None if BLOCK_DRAM_BYTES_PER_LAUNCH is None else BLOCK_DRAM_BYTES_PER_LAUNCH * cfg.num_layers
    dom_ms = _time_graph(graph, max(5, args.steps // 2))
    achieved = dom_bytes / (dom_ms / 1000) / 1e9
    round_achieved = bytes_["total"] / (ms_per_step / 1000) / 1e9
    del graph, keep

    # End to end through the public API: configs[2]'s requests (256-token random prompts, 512 new tokens, seeds 0, 1,
    # 2 in turn), a contiguous slice of the job's request list per rank; the job's time is the slowest rank's.
    per_rank = 0 if args.skip_e2e else args.e2e_requests
    e2e_tokens, e2e_rounds, e2e_s = 0, 0, 0.0
    if per_rank:
        requests = [(i, i % 3) for i in range(rank * per_rank, (rank + 1) * per_rank)]  # (prompt index, seed)
        prompts = {i: torch.randint(0, cfg.vocab, (PROMPT_E2E,), generator=torch.Generator().manual_seed(1000 + i))
                   .pin_memory() for i, _ in requests}
        decoder.generate(prompts[requests[0][0]], TOKENS_E2E, seed=0, stop_at_eos=False)  # warm-up request
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for i, seed in requests:
            res = decoder.generate(prompts[i], TOKENS_E2E, seed=seed, stop_at_eos=False)
            e2e_tokens += len(res.token_ids)
            e2e_rounds += res.steady_rounds
        e2e_s = time.perf_counter() - t0
        e2e_s, e2e_tokens = reduce_over_ranks(dist, e2e_s, e2e_tokens)
    e2e_value = e2e_tokens / e2e_s if e2e_s else None

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:  # the CPU baseline is an N=1 figure
        _seed_context(decoder, cfg, ctx=args.ctx)
        cpu = cpu_baseline(weights, decoder, cfg, rounds=1)

    if rank == 0:
        # prologue, per layer qkv + attention + (block | o, norm, gate_up, down) + norm, then lm_head and verify
        launches_per_round = 1 + (7 if args.separate_mlp else 4) * cfg.num_layers + 2
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args.ctx, world), "ctx_mean": ctx_mean,
            "round_us": 1000 * ms_per_step,
            "tokens_per_round": total_tokens / (args.steps * world),
            "roofline": {"bound": "hbm", "kernel": dom_kernel,
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": dom_traffic,
                         "traffic_prefetch": None if args.separate_mlp else
                         BLOCK_PREFETCH_BYTES_PER_LAUNCH * cfg.num_layers,
                         "bytes_per_round": dom_bytes,
                         "ms_per_round": dom_ms, "launches_per_round": dom_launches},
            "round_roofline": {"bound": "hbm", "achieved": round_achieved, "peak": peak, "unit": "GB/s",
                               "frac": round_achieved / peak, "bytes_per_round": bytes_},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": PROMPT_E2E * 8,
                    "d2h_bytes_per_step": int(e2e_rounds / max(per_rank, 1)) * 16 + TOKENS_E2E * 8,
                    "step": f"one request: {PROMPT_E2E}-token prompt, {TOKENS_E2E} new tokens (BASELINE configs[2], "
                            f"seeds 0, 1, 2 in turn)", "requests": per_rank * world,
                    "sharding": "a contiguous slice of the request list per rank"},
            "cpu_baseline": cpu,
            "gpu_launches": launches_per_round * args.steps,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line))
    decoder.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", default="native", choices=("native", "reference", "reference-gpu"),
                        help="reference: the CPU round oracle (the reference has no CPU round path); reference-gpu: "
                             "the reference's own vLLM round from baseline/_ref beside this engine's, on one GPU")
    parser.add_argument("--skip-cpu", action="store_true", help="omit the CPU oracle baseline")
    parser.add_argument("--skip-e2e", action="store_true", help="omit the end-to-end requests (profiling runs)")
    parser.add_argument("--ctx", type=int, default=CTX, help="committed context of the timed rounds (tokens)")
    parser.add_argument("--e2e-requests", type=int, default=2,
                        help="end-to-end requests per rank (configs[2] runs 64 in all: --e2e-requests 64/N)")
    parser.add_argument("--separate-mlp", action="store_true",
                        help="gate_up and down as two launches instead of the persistent MLP block launch")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
