"""The reference's own round on the GPU, for comparison on the same box (child process of
``bench.py --impl reference-gpu``; not part of the native engine).

    PYTHONPATH=baseline/_ref python plm-anon_b200/bench/reference_gpu.py <export dir> <default|fast> <seed> <tokens>

Runs justuswill/PLM-anon as installed into baseline/_ref (its plm.rounds.RoundConfig -> vLLM RoundDecoder, with
``--mode default``: cuBLAS and Inductor FlexAttention, or ``--mode fast``: its Triton split-K GEMM tiles), on a
256-token prompt of the export's word-level tokenizer, exact match, k = 7, 16-token pages, and prints one JSON line:
the second of two requests (the first pays compilation and graph capture).
"""

from __future__ import annotations

import json
import os
import sys
import time


def main() -> None:
    model, mode, seed, tokens = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4])
    os.environ.setdefault("HF_HUB_OFFLINE", "1")
    os.environ.setdefault("TRANSFORMERS_OFFLINE", "1")
    import torch
    import plm
    from plm.rounds import RoundConfig

    if "baseline" not in plm.__file__:
        raise SystemExit(f"expected the reference's installed package, found {plm.__file__}")
    started = time.perf_counter()
    decoder = RoundConfig(model=model, setting="posttrain", mode=mode, match="exact", k=7, dtype="bfloat16",
                          max_model_len=2048).build(0.5, 1 << 30, 16)
    build_s = time.perf_counter() - started
    vocab = decoder.vocab
    ids = torch.randint(0, vocab, (256,), generator=torch.Generator().manual_seed(seed))
    prompt = " ".join(f"w{int(i)}" for i in ids)
    decoder.generate(prompt, 64, seed=0, stop_at_eos=False)
    res = decoder.generate(prompt, tokens, seed=0, stop_at_eos=False)
    print(json.dumps({"impl": f"reference --mode {mode}", "package": plm.__file__, "build_s": build_s,
                      "steady_rounds": res.steady_rounds, "steady_ms": res.steady_ms,
                      "round_us": 1000.0 * res.steady_ms / max(res.steady_rounds, 1), "tokens": len(res.token_ids),
                      "seconds": res.seconds, "tokens_per_second": len(res.token_ids) / res.seconds}))


if __name__ == "__main__":
    main()
