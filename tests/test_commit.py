"""The KV commit of a round (plm_commit, and inside plm_round / plm_round0) on the GPU.

BASELINE configs[4]'s cache-management sweep: contexts 512-32768, k in {4, 6, 7, 8}, pages of 16 and 32 tokens (and
the reference's 64), block tables with 0-90% of the pool's pages left free in between, and an accepted count per
round drawn uniformly from [0, k] (so 1 .. k committed rows per round; acceptance never commits more than the k
verify rows). Every round's scratch rows are random bf16; the cache must equal the oracle's commit bit for bit, and
every slot outside the committed rows must keep its previous contents.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rounds as orounds

pytestmark = pytest.mark.gpu


def _fragmented_table(max_pages: int, fragmentation: float, rng: np.random.Generator) -> tuple[np.ndarray, int]:
    """A block table of max_pages pages spread over a pool in which about ``fragmentation`` of the pages lie free
    between the used ones (the used pages in a random order)."""
    pool = int(np.ceil(max_pages / (1.0 - fragmentation))) if fragmentation < 1 else max_pages
    used = np.sort(rng.choice(pool, size=max_pages, replace=False))
    return rng.permutation(used).astype(np.int32), pool


@pytest.mark.parametrize("ctx_len,k,page,fragmentation", [
    (512, 4, 16, 0.0),
    (1024, 7, 16, 0.5),
    (4096, 6, 32, 0.9),
    (32768, 8, 16, 0.3),
    (2000, 7, 64, 0.7),
    (777, 8, 32, 0.1),
])
def test_commit_sweep_bit_exact(ctx, ctx_len, k, page, fragmentation):
    from plm import native

    rng = np.random.default_rng(ctx_len + 31 * k + page)
    layers, kv_heads, hd, rounds = 2, 4, 128, 12
    width = k + k * k
    max_pages = -(-(ctx_len + rounds * k + width) // page) + 1
    table, num_pages = _fragmented_table(max_pages, fragmentation, rng)
    cache = (torch.randn(layers, 2, num_pages, kv_heads, page, hd, device="cuda")).bfloat16()
    expect = cache.view(torch.int16).cpu().numpy().copy()
    table_t = torch.as_tensor(table, device="cuda")
    record = torch.zeros(2, dtype=torch.int64, device="cuda")
    scratch = torch.empty(layers, 2, width, kv_heads, hd, dtype=torch.bfloat16, device="cuda")
    offset = ctx_len
    for _ in range(rounds):
        nc = int(rng.integers(0, k))  # accepted proposals 0 .. k-1: nc + 1 verify rows are committed
        scratch.copy_(torch.randn(scratch.shape, device="cuda").bfloat16())
        record.copy_(torch.tensor([offset, nc + 1]))
        desc = native.CommitDesc(dtype=native.PLM_BF16, scratch=scratch.data_ptr(), scratch_rows=width,
                                 kv_cache=cache.data_ptr(), plane_elems=num_pages * kv_heads * page * hd,
                                 layers=layers, num_kv_heads=kv_heads, head_dim=hd, page_size=page,
                                 num_pages=num_pages, max_pages=max_pages, block_table=table_t.data_ptr(),
                                 commit=record.data_ptr())
        native.commit(ctx, desc)
        orounds.commit_rows(expect, scratch.view(torch.int16).cpu().numpy(), table, page, offset, nc + 1)
        offset += nc + 1
    ctx.check()
    np.testing.assert_array_equal(cache.view(torch.int16).cpu().numpy(), expect)


def test_commit_rejects_bad_pages(ctx):
    """A commit record that reaches past the block table is skipped and reported, not written anywhere."""
    from plm import native

    layers, kv_heads, hd, page, max_pages = 1, 2, 64, 16, 4
    cache = torch.zeros(layers, 2, max_pages, kv_heads, page, hd, dtype=torch.bfloat16, device="cuda")
    scratch = torch.ones(layers, 2, 8, kv_heads, hd, dtype=torch.bfloat16, device="cuda")
    table = torch.arange(max_pages, dtype=torch.int32, device="cuda")
    record = torch.tensor([max_pages * page - 2, 4], dtype=torch.int64, device="cuda")
    desc = native.CommitDesc(dtype=native.PLM_BF16, scratch=scratch.data_ptr(), scratch_rows=8,
                             kv_cache=cache.data_ptr(), plane_elems=max_pages * kv_heads * page * hd, layers=layers,
                             num_kv_heads=kv_heads, head_dim=hd, page_size=page, num_pages=max_pages,
                             max_pages=max_pages, block_table=table.data_ptr(), commit=record.data_ptr())
    native.commit(ctx, desc)
    with pytest.raises(native.NativeError):
        ctx.check()
    written = cache[:, :, max_pages - 1, :, page - 2:, :]  # logical 62 and 63: the two rows inside the table
    assert written.eq(1).all().item()
    assert cache.float().abs().sum().item() == written.numel()  # nothing else was written


def test_round_commits_only_the_accepted_verify_rows():
    """Inside the round: after each steady round the cache holds, at logical offset .. offset + nc, exactly rows
    0 .. nc of the round's scratch (the verify rows), and no other slot of the pool changed: the proposal rows,
    the selected block among them, stay out of the committed context."""
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    cfg = shape_config("plm-tiny")
    decoder = RoundDecoder(PLMWeights.random(cfg, seed=3), 7, block_size=16, kv_cache_bytes=64 << 20,
                           max_model_len=1024)
    prompt = torch.randint(0, cfg.vocab, (50,), generator=torch.Generator().manual_seed(2))
    decoder.handle.load_prompt(prompt.pin_memory())
    decoder.handle.prefill()
    decoder.handle.round0()
    torch.cuda.synchronize()
    st = decoder.handle.state()
    from plm import native

    width, kvh, hd = decoder.width, cfg.num_kv_heads, cfg.head_dim
    round_kv = native.device_view(st.round_kv, (cfg.num_layers, 2, width, kvh, hd), torch.bfloat16)
    record = native.device_view(st.commit, (2,), torch.int64)
    table = native.device_view(st.block_table, (decoder.max_pages,), torch.int32).cpu().numpy()
    committed_rows = 0
    for _ in range(6):
        before = decoder.kv_cache.view(torch.int16).cpu().numpy().copy()
        offset = int(decoder.offset_t)
        decoder.handle.round()
        torch.cuda.synchronize()
        first, count = record.tolist()
        assert first == offset and count == int(decoder.offset_t) - offset >= 1
        orounds.commit_rows(before, round_kv.view(torch.int16).cpu().numpy(), table, 16, first, count)
        np.testing.assert_array_equal(decoder.kv_cache.view(torch.int16).cpu().numpy(), before)
        committed_rows += count
    decoder.check()
    assert committed_rows >= 6
    decoder.close()
