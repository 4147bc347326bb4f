"""plm_attention and plm_kv_append on the GPU.

Attention is compared with a plain PyTorch fp32 reference of the same op: keys gathered through the block table,
the round mask of plm/mask.py:23-29 (oracle.rounds.visible), softmax, P.V. Tolerance: the kernel rounds P to bf16
before P.V and the output once to bf16, so |err| <= 2e-2 * max|ref| + 1e-2 (outputs are O(1)).
KV append must reproduce the cache contents bit for bit (a pure scatter).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import rounds as orounds

pytestmark = pytest.mark.gpu


def _layout(kind: str, k: int, rows: int):
    if kind == "steady":
        _, _, depth, own = orounds.steady_layout(k)
    elif kind == "round0":
        _, _, depth, own = orounds.round0_layout(k)
    else:
        _, _, depth, own = orounds.chunk_layout(rows)
    return depth, own


def _pool(num_pages, kv_heads, page, hd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(num_pages, kv_heads, page, hd, generator=g, device="cuda").bfloat16()
    v = torch.randn(num_pages, kv_heads, page, hd, generator=g, device="cuda").bfloat16()
    return k, v


def _reference(q, kc, vc, table, offset, depth, own, page, heads, kv_heads):
    rows, hd = q.shape[0], q.shape[-1]
    n_keys = offset + rows
    logical = torch.arange(n_keys, device="cuda")
    pages = table.long()[logical // page]
    keys = kc[pages, :, logical % page, :].float().repeat_interleave(heads // kv_heads, dim=1)
    vals = vc[pages, :, logical % page, :].float().repeat_interleave(heads // kv_heads, dim=1)
    mask = torch.as_tensor(orounds.visible(depth, own, offset, n_keys), device="cuda")
    s = torch.einsum("rhd,khd->hrk", q.float(), keys) / math.sqrt(hd)
    s = s.masked_fill(~mask[None], float("-inf"))
    return torch.einsum("hrk,khd->rhd", torch.softmax(s, dim=-1), vals)


@pytest.mark.parametrize("kind,k,ctx_len,page,heads,kv_heads,hd,splits", [
    ("steady", 7, 1024, 16, 16, 16, 128, 0),
    ("steady", 7, 4096, 16, 16, 16, 128, 0),
    ("steady", 7, 32768, 16, 16, 16, 128, 0),   # the longest context of the configs[4] sweep
    ("steady", 7, 4096, 64, 16, 16, 128, 0),    # the reference's page size (bench/engine.py:4)
    ("steady", 7, 4096, 16, 20, 20, 128, 0),    # the 3B shape's 20 heads
    # 16 splits: two clusters of 8 per head merged through memory (the second idle below 64 key tiles)
    ("steady", 7, 4096, 16, 16, 16, 128, 16),
    ("steady", 7, 32768, 16, 16, 16, 128, 16),
    ("steady", 7, 1024, 16, 16, 16, 128, 16),
    ("steady", 7, 8192, 32, 16, 4, 128, 16),
    ("steady", 7, 1000, 32, 16, 16, 128, 1),
    ("steady", 4, 333, 64, 8, 8, 64, 0),
    ("steady", 6, 190, 16, 8, 8, 64, 2),
    ("steady", 8, 2048, 16, 16, 4, 128, 0),
    ("round0", 7, 256, 16, 16, 16, 128, 0),
    ("chunk", 0, 0, 16, 16, 16, 128, 0),
    ("chunk", 0, 512, 32, 8, 8, 64, 0),
    # split counts that are not powers of two: each cluster rank combines ceil(64 / splits) rows, the last fewer
    ("steady", 7, 1024, 16, 16, 16, 128, 7),
    ("chunk", 0, 512, 16, 16, 16, 128, 7),      # full 64-row query tiles: row 63 lies in the last rank's share
    ("chunk", 0, 300, 32, 8, 8, 64, 5),
    ("steady", 6, 190, 16, 8, 8, 64, 3),
])
def test_attention_matches_fp32(ctx, kind, k, ctx_len, page, heads, kv_heads, hd, splits):
    from plm import native

    rows = k + k * k if kind != "chunk" else 200
    depth, own = _layout(kind, k, rows)
    total = ctx_len + rows
    max_pages = -(-total // page) + 2
    num_pages = max_pages * 2
    g = torch.Generator(device="cuda").manual_seed(7)
    table = torch.randperm(num_pages, generator=g, device="cuda")[:max_pages].to(torch.int32).contiguous()
    kc, vc = _pool(num_pages, kv_heads, page, hd, seed=8)
    q = torch.randn(rows, heads, hd, generator=g, device="cuda").bfloat16().contiguous()
    out = torch.full((rows, heads * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    offset = torch.tensor([ctx_len], dtype=torch.int64, device="cuda")
    depth_t = torch.as_tensor(depth, dtype=torch.int32, device="cuda")
    own_t = torch.as_tensor(own, dtype=torch.int32, device="cuda")
    desc = native.AttentionDesc(dtype=native.PLM_BF16, q=q.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
                                block_table=table.data_ptr(), max_pages=max_pages, num_pages=num_pages,
                                page_size=page, offset=offset.data_ptr(), rows=rows, depth=depth_t.data_ptr(),
                                own_start=own_t.data_ptr(), num_heads=heads, num_kv_heads=kv_heads, head_dim=hd,
                                out=out.data_ptr(), splits=splits, max_keys=total)
    native.attention(ctx, desc)
    ctx.check()
    ref = _reference(q, kc, vc, table, ctx_len, depth, own, page, heads, kv_heads).reshape(rows, heads * hd)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, f"max abs err {err}"


def test_attention_split_invariance(ctx):
    """Any split count gives the same answer within fp32 reassociation; one split count is bit-reproducible."""
    from plm import native

    k, ctx_len, page, heads, hd = 7, 2000, 16, 16, 128
    rows = k + k * k
    depth, own = _layout("steady", k, rows)
    max_pages = -(-(ctx_len + rows) // page)
    kc, vc = _pool(max_pages, heads, page, hd, seed=9)
    table = torch.arange(max_pages, dtype=torch.int32, device="cuda")
    q = torch.randn(rows, heads, hd, device="cuda").bfloat16()
    offset = torch.tensor([ctx_len], dtype=torch.int64, device="cuda")
    depth_t = torch.as_tensor(depth, dtype=torch.int32, device="cuda")
    own_t = torch.as_tensor(own, dtype=torch.int32, device="cuda")
    outs = {}
    for splits in (1, 4, 7, 8, 8):
        out = torch.zeros(rows, heads * hd, dtype=torch.bfloat16, device="cuda")
        desc = native.AttentionDesc(dtype=native.PLM_BF16, q=q.data_ptr(), k_cache=kc.data_ptr(),
                                    v_cache=vc.data_ptr(), block_table=table.data_ptr(), max_pages=max_pages,
                                    num_pages=max_pages, page_size=page, offset=offset.data_ptr(), rows=rows,
                                    depth=depth_t.data_ptr(), own_start=own_t.data_ptr(), num_heads=heads,
                                    num_kv_heads=heads, head_dim=hd, out=out.data_ptr(), splits=splits,
                                    max_keys=ctx_len + rows)
        native.attention(ctx, desc)
        ctx.check()
        if splits in outs:
            assert torch.equal(outs[splits], out)
        outs[splits] = out
    for splits in (4, 7, 8):
        assert (outs[splits].float() - outs[1].float()).abs().max().item() < 2e-2


def test_attention_sixteen_splits_need_resident_clusters(ctx):
    """16 splits wait for one another, so a launch whose clusters cannot all be resident at once (k = 8: 72 rows in
    two query tiles, 64 clusters of 8) is refused up front instead of risking a wait."""
    from plm import native

    k, ctx_len, page, heads, hd = 8, 4096, 16, 16, 128
    rows = k + k * k
    depth, own = _layout("steady", k, rows)
    max_pages = -(-(ctx_len + rows) // page)
    kc, vc = _pool(max_pages, heads, page, hd, seed=11)
    table = torch.arange(max_pages, dtype=torch.int32, device="cuda")
    q = torch.randn(rows, heads, hd, device="cuda").bfloat16()
    out = torch.zeros(rows, heads * hd, dtype=torch.bfloat16, device="cuda")
    offset = torch.tensor([ctx_len], dtype=torch.int64, device="cuda")
    depth_t = torch.as_tensor(depth, dtype=torch.int32, device="cuda")
    own_t = torch.as_tensor(own, dtype=torch.int32, device="cuda")
    desc = native.AttentionDesc(dtype=native.PLM_BF16, q=q.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(),
                                block_table=table.data_ptr(), max_pages=max_pages, num_pages=max_pages,
                                page_size=page, offset=offset.data_ptr(), rows=rows, depth=depth_t.data_ptr(),
                                own_start=own_t.data_ptr(), num_heads=heads, num_kv_heads=heads, head_dim=hd,
                                out=out.data_ptr(), splits=16, max_keys=ctx_len + rows)
    with pytest.raises(native.NativeError, match="resident"):
        native.attention(ctx, desc)


def test_attention_two_cluster_merge_invariance(ctx):
    """16 splits (two clusters merged through memory) agree with 8 within fp32 reassociation and repeat bit for
    bit, launch after launch (the merge counters return to zero)."""
    from plm import native

    k, ctx_len, page, heads, hd = 7, 5000, 16, 16, 128
    rows = k + k * k
    depth, own = _layout("steady", k, rows)
    max_pages = -(-(ctx_len + rows) // page)
    kc, vc = _pool(max_pages, heads, page, hd, seed=10)
    table = torch.arange(max_pages, dtype=torch.int32, device="cuda")
    q = torch.randn(rows, heads, hd, device="cuda").bfloat16()
    offset = torch.tensor([ctx_len], dtype=torch.int64, device="cuda")
    depth_t = torch.as_tensor(depth, dtype=torch.int32, device="cuda")
    own_t = torch.as_tensor(own, dtype=torch.int32, device="cuda")
    outs = []
    for splits in (8, 16, 16, 16):
        out = torch.zeros(rows, heads * hd, dtype=torch.bfloat16, device="cuda")
        desc = native.AttentionDesc(dtype=native.PLM_BF16, q=q.data_ptr(), k_cache=kc.data_ptr(),
                                    v_cache=vc.data_ptr(), block_table=table.data_ptr(), max_pages=max_pages,
                                    num_pages=max_pages, page_size=page, offset=offset.data_ptr(), rows=rows,
                                    depth=depth_t.data_ptr(), own_start=own_t.data_ptr(), num_heads=heads,
                                    num_kv_heads=heads, head_dim=hd, out=out.data_ptr(), splits=splits,
                                    max_keys=ctx_len + rows)
        native.attention(ctx, desc)
        ctx.check()
        outs.append(out)
    assert torch.equal(outs[1], outs[2]) and torch.equal(outs[1], outs[3])
    assert (outs[1].float() - outs[0].float()).abs().max().item() < 2e-2


def test_attention_permutation_invariance(ctx):
    """Results do not depend on where pages live: a shuffled pool with the matching table gives identical bits."""
    from plm import native

    k, ctx_len, page, heads, hd = 7, 700, 16, 8, 64
    rows = k + k * k
    depth, own = _layout("steady", k, rows)
    n = -(-(ctx_len + rows) // page)
    kc, vc = _pool(n, heads, page, hd, seed=10)
    perm = torch.randperm(n, device="cuda")
    kc2, vc2 = torch.empty_like(kc), torch.empty_like(vc)
    kc2[perm] = kc
    vc2[perm] = vc
    q = torch.randn(rows, heads, hd, device="cuda").bfloat16()
    offset = torch.tensor([ctx_len], dtype=torch.int64, device="cuda")
    depth_t = torch.as_tensor(depth, dtype=torch.int32, device="cuda")
    own_t = torch.as_tensor(own, dtype=torch.int32, device="cuda")
    results = []
    for table, kk, vv in ((torch.arange(n, dtype=torch.int32, device="cuda"), kc, vc), (perm.to(torch.int32), kc2, vc2)):
        out = torch.zeros(rows, heads * hd, dtype=torch.bfloat16, device="cuda")
        desc = native.AttentionDesc(dtype=native.PLM_BF16, q=q.data_ptr(), k_cache=kk.data_ptr(), v_cache=vv.data_ptr(),
                                    block_table=table.contiguous().data_ptr(), max_pages=n, num_pages=n, page_size=page,
                                    offset=offset.data_ptr(), rows=rows, depth=depth_t.data_ptr(),
                                    own_start=own_t.data_ptr(), num_heads=heads, num_kv_heads=heads, head_dim=hd,
                                    out=out.data_ptr(), splits=4, max_keys=ctx_len + rows)
        native.attention(ctx, desc)
        ctx.check()
        results.append(out)
    assert torch.equal(results[0], results[1])


@pytest.mark.parametrize("page,fragmentation,k,ctx_len", [(16, 0.0, 7, 512), (16, 0.9, 4, 4000), (32, 0.5, 8, 32700),
                                                          (32, 0.3, 6, 1000)])
def test_kv_append_bit_exact(ctx, page, fragmentation, k, ctx_len):
    """Cache contents after appending a round's rows equal a numpy scatter through the same block table
    (a fragmented pool: a fraction of pages interleaved as occupied by other requests)."""
    from plm import native

    rows, kv_heads, hd = k + k * k, 16, 128
    rng = np.random.default_rng(int(fragmentation * 100) + page)
    need = -(-(ctx_len + rows) // page)
    num_pages = int(need / max(1e-9, 1 - fragmentation)) + 4
    table = rng.permutation(num_pages)[:need].astype(np.int32)
    kc = torch.zeros(num_pages, kv_heads, page, hd, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    g = torch.Generator(device="cuda").manual_seed(11)
    kr = torch.randn(rows, kv_heads, hd, generator=g, device="cuda").bfloat16()
    vr = torch.randn(rows, kv_heads, hd, generator=g, device="cuda").bfloat16()
    table_d = torch.as_tensor(table, device="cuda")
    offset = torch.tensor([ctx_len], dtype=torch.int64, device="cuda")
    desc = native.KvAppendDesc(dtype=native.PLM_BF16, k=kr.data_ptr(), v=vr.data_ptr(), k_cache=kc.data_ptr(),
                               v_cache=vc.data_ptr(), block_table=table_d.data_ptr(), max_pages=need,
                               num_pages=num_pages, page_size=page, offset=offset.data_ptr(), rows=rows,
                               num_kv_heads=kv_heads, head_dim=hd)
    native.kv_append(ctx, desc)
    ctx.check()
    expect_k = np.zeros((num_pages, kv_heads, page, hd), dtype=np.uint16)
    expect_v = np.zeros_like(expect_k)
    logical = ctx_len + np.arange(rows)
    pages, slots = table[logical // page], logical % page
    expect_k[pages, :, slots, :] = kr.view(torch.int16).cpu().numpy().view(np.uint16)
    expect_v[pages, :, slots, :] = vr.view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(kc.view(torch.int16).cpu().numpy().view(np.uint16), expect_k)
    np.testing.assert_array_equal(vc.view(torch.int16).cpu().numpy().view(np.uint16), expect_v)
