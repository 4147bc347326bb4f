"""Host-side logic on CPU: the drop-in configuration surface (plm/rounds.py of the reference), model configuration and
export round trip, the roofline byte accounting of bench.py, and the multi-GPU timing reduction (gloo, 2 ranks)."""

from __future__ import annotations

import os
import socket

import pytest
import torch


def test_round_config_matches_reference_settings():
    from plm.rounds import PREFILL_BUCKETS, SETTINGS, RoundConfig

    assert PREFILL_BUCKETS == tuple(range(64, 641, 64))
    assert SETTINGS["posttrain"].default_k == {"exact": 7, "relaxed": 10}
    assert SETTINGS["pretrain"].relaxed_rule == ("floor", 2e-3)
    c = RoundConfig(model="synthetic:plm-tiny")
    assert (c.k, c.width, c.accept) == (7, 56, ("nucleus", None))
    c = RoundConfig(model="x", setting="posttrain", match="relaxed")
    assert (c.k, c.accept) == (10, ("nucleus", 0.94))
    c = RoundConfig(model="x", setting="pretrain", match="relaxed")
    assert (c.k, c.accept, c.width) == (6, ("floor", 2e-3), 42)
    c = RoundConfig(model="x", setting="pretrain", k=4)
    assert c.describe()["accept"] == "exact" and c.describe()["width"] == 20
    with pytest.raises(ValueError):
        RoundConfig(model="x", setting="other")
    with pytest.raises(ValueError):
        RoundConfig(model="x", match="loose")


def test_config_and_export_round_trip(tmp_path):
    from plm.model import PLMConfig, PLMWeights, shape_config

    cfg = shape_config("plm-tiny", vocab=1000, aux_vocab=64, num_kv_heads=1)
    assert PLMConfig.from_hf_config(cfg.hf_config(), name=cfg.name) == cfg
    w = PLMWeights.random(cfg, seed=3, device="cpu")
    w.save_export(tmp_path / "export")
    back = PLMWeights.from_export(tmp_path / "export", device="cpu")
    for name, value in w.named().items():
        other = back.named()[name]
        if isinstance(value, list):
            assert all(torch.equal(a, b) for a, b in zip(value, other)), name
        else:
            assert torch.equal(value, other), name
    again = PLMWeights.random(cfg, seed=3, device="cpu")
    assert torch.equal(again.qkv[1], w.qkv[1]) and not torch.equal(PLMWeights.random(cfg, seed=4, device="cpu").o[0],
                                                                   w.o[0])


def test_roofline_bytes_of_the_benchmark_shape():
    from plm.model import shape_config

    bench = _load_root_bench()
    b = bench.round_bytes(shape_config("plm-1.3b"), 1024, 7)
    assert b["weights"] == 3_427_078_144  # 24 layers of qkv/o/gate_up/down + lm_head, bf16
    assert b["kv_read"] == 1024 * 24 * 2 * 2048 * 2
    assert abs(b["total"] / 1e9 - 3.65) < 0.01


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _load_root_bench():
    """bench.py at the repository root (the name ``bench`` also belongs to the CLI package)."""
    import importlib.util
    from pathlib import Path

    path = Path(__file__).resolve().parent.parent / "bench.py"
    spec = importlib.util.spec_from_file_location("plm_root_bench", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    bench = _load_root_bench()

    elapsed, tokens = bench.reduce_over_ranks(dist, 10.0 + rank, 100 + rank, device="cpu")
    queue.put((rank, elapsed, tokens))
    dist.barrier()
    dist.destroy_process_group()


def test_multi_rank_reduction_gloo():
    """Replicas only: the job time is the slowest rank's, the token count the sum over ranks."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, elapsed, tokens in results:
        assert elapsed == 11.0 and tokens == 201


def test_generate_cli_surface(tmp_path):
    """bench.generate / bench.harness: the reference's flags parse, datasets load (token-id lists and the random
    spec), per-pass aggregates follow bench/harness.py:33-39, and the baselines outside the round path exit."""
    import argparse
    import json

    from tests.conftest import cli_bench

    generate, harness = cli_bench()

    parser = argparse.ArgumentParser()
    generate.add_arguments(parser)
    harness.add_run_arguments(parser)
    args = parser.parse_args(["--model", "synthetic:plm-tiny", "--match", "relaxed", "--setting", "pretrain",
                              "--dataset", "random:3:16:5", "--tokens", "32", "--seeds", "0", "1"])
    assert (args.match, args.setting, args.k, args.seeds, args.tokens) == ("relaxed", "pretrain", None, [0, 1], 32)
    ds = harness.load_dataset(args.dataset, 2, vocab=1000)
    assert len(ds) == 2 and all(len(p) == 16 and max(p) < 1000 for p in ds)
    assert ds == harness.load_dataset("random:3:16:5", 2, vocab=1000)
    path = tmp_path / "prompts.json"
    path.write_text(json.dumps([[1, 2, 3], "text"]))
    assert harness.load_dataset(str(path), None) == [[1, 2, 3], "text"]
    path.write_text(json.dumps({"not": "a list"}))
    with pytest.raises(SystemExit):
        harness.load_dataset(str(path), None)
    records = [harness.speed_record("p", "", [1, 2], 2, 10, 100.0, 40.0, 8),
               harness.speed_record("q", "", [0], 1, 5, 50.0, 20.0, 3)]
    agg = harness.aggregate(records)
    assert agg["calls"] == 3 and agg["tokens"] == 15
    assert abs(agg["tokens_per_second"] - 1000 * 15 / 60.0) < 1e-9
    assert abs(agg["e2e_tokens_per_second"] - 1000 * 15 / 150.0) < 1e-9
    args.ar = True
    rc = generate.round_config(args)  # AR-Voronoi: exact matching, one verify row per step
    assert (rc.k, rc.match, rc.width) == (1, "exact", 2)
    args.ar_sampler = "topk"
    with pytest.raises(SystemExit):
        generate.build_generator(args)
    args.ar, args.fdv2 = False, True
    with pytest.raises(SystemExit):
        generate.build_generator(args)


def test_float16_export_keeps_its_dtype(tmp_path):
    """A float16 export loads as float16 (never relabelled as bfloat16); a dtype is converted only when asked for,
    and RoundConfig takes the export's own dtype unless one is given."""
    from plm.model import PLMWeights, shape_config
    from plm.rounds import RoundConfig

    cfg = shape_config("plm-tiny", vocab=1000, aux_vocab=64, dtype="float16")
    w = PLMWeights.random(cfg, seed=1, device="cpu")
    export = w.save_export(tmp_path / "fp16")
    kept = PLMWeights.from_export(export, device="cpu")
    assert kept.config.dtype == "float16" and kept.embed.dtype == torch.float16 and kept.qkv[0].dtype == torch.float16
    assert torch.equal(kept.qkv[1], w.qkv[1])
    converted = PLMWeights.from_export(export, device="cpu", dtype="bfloat16")
    assert converted.config.dtype == "bfloat16" and converted.o[0].dtype == torch.bfloat16
    assert torch.equal(converted.o[0], w.o[0].bfloat16())
    assert RoundConfig(model=str(export)).dtype == "float16"
    assert RoundConfig(model=str(export), dtype="bfloat16").dtype == "bfloat16"
    assert RoundConfig(model="synthetic:plm-tiny").dtype == "bfloat16"


def test_oracle_commit_moves_rows_through_the_block_table():
    """oracle.rounds.commit_rows on a hand-checked case: rows go to logical first .. first + count - 1, each to
    its page through the block table, in both planes of every layer, and nothing else changes."""
    import numpy as np

    from oracle import rounds as orounds

    cache = np.zeros((2, 2, 3, 1, 4, 2), dtype=np.int16)  # layers, K|V, pages, kv heads, page size 4, head dim
    scratch = np.arange(2 * 2 * 5 * 1 * 2, dtype=np.int16).reshape(2, 2, 5, 1, 2) + 1
    orounds.commit_rows(cache, scratch, np.array([2, 0, 1]), 4, 3, 3)
    np.testing.assert_array_equal(cache[:, :, 2, :, 3, :], scratch[:, :, 0])  # logical 3 -> page 2, slot 3
    np.testing.assert_array_equal(cache[:, :, 0, :, 0, :], scratch[:, :, 1])  # logical 4 -> page 0, slot 0
    np.testing.assert_array_equal(cache[:, :, 0, :, 1, :], scratch[:, :, 2])  # logical 5 -> page 0, slot 1
    assert np.count_nonzero(cache) == np.count_nonzero(scratch[:, :, :3])


def test_timeline_critical_path_adds_up_to_the_span():
    """bench/timeline.py's accounting on synthetic kernel records of two rounds: a launch's critical path is the time
    from the previous launch's end to its own, overlapping launches (programmatic dependent launch) included, and the
    critical paths of a round add up to its span; the last GEMM of a round is lm_head."""
    import importlib.util
    from pathlib import Path

    path = Path(__file__).resolve().parents[1] / "plm-anon_b200" / "bench" / "timeline.py"
    spec = importlib.util.spec_from_file_location("plm_timeline", path)
    tl = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tl)
    one_round = [("embed_norm_kernel", 0, 4), ("skinny_gemm_kernel<2>", 3, 15), ("round_attention_kernel", 14, 16),
                 ("mlp_block_kernel", 20, 44), ("add_norm_kernel", 60, 8), ("skinny_gemm_kernel<3>", 66, 40),
                 ("verify_decode_kernel", 106, 110), ("commit_kernel", 214, 4)]
    events = []
    for r in range(2):
        events += [{"name": n, "ts": 1000 * r + t, "dur": d, "cat": "kernel"} for n, t, d in one_round]
    result = tl.summarise(events, rounds=2)
    assert result["launches"] == len(one_round)
    assert result["span_us"] == 218.0
    crit = [x["critical_us"] for x in result["timeline"]]
    assert crit == [4, 14, 12, 34, 4, 38, 110, 2]
    assert abs(sum(crit) - result["span_us"]) < 1e-9
    kinds = result["kinds"]
    assert kinds["skinny_gemm (qkv)"]["launches"] == 1 and kinds["skinny_gemm (lm_head)"]["launches"] == 1
    assert abs(sum(v["critical_share"] for v in kinds.values()) - 1.0) < 5e-3  # shares rounded to 3 places
