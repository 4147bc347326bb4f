"""plm_gemm (tcgen05 skinny GEMM) against a plain PyTorch fp32 reference of the same op, for every fused epilogue.

Tolerance: the kernel accumulates in fp32 and rounds once to bf16, so each output is within one bf16 rounding
(relative 2^-8) of the fp32 reference plus accumulation-order noise; checked as rtol 8e-3, atol 1e-3 * max|ref|.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


def _close(actual, expected):
    atol = 1e-3 * float(expected.abs().max()) + 1e-6
    torch.testing.assert_close(actual.float(), expected.float(), rtol=8e-3, atol=atol)


@pytest.mark.parametrize("n_out,k,rows", [
    (6144, 2048, 56), (2048, 2048, 56), (2048, 8192, 56), (16384, 2048, 56),
    (1536, 512, 42), (512, 2048, 42), (384, 256, 16), (200, 128, 7), (2560, 2560, 56), (768, 640, 72),
    (1024, 512, 128), (640, 1024, 256), (1024, 512, 110), (256, 256, 20),
])
def test_store_matches_fp32(ctx, n_out, k, rows):
    from plm import native

    w = _rand(n_out, k, scale=0.02, seed=1)
    x = _rand(rows, k, seed=2)
    out = torch.full((rows, n_out), float("nan"), dtype=torch.bfloat16, device="cuda")
    native.gemm(ctx, w, x, rows, out=out)
    ctx.check()
    ref = x.float() @ w.float().T
    _close(out, ref)


@pytest.mark.parametrize("splits", [1, 2, 3, 4, 5, 8])
def test_forced_splits_and_determinism(ctx, splits):
    from plm import native

    w = _rand(1024, 2048, scale=0.02, seed=3)
    x = _rand(56, 2048, seed=4)
    outs = []
    for _ in range(2):
        out = torch.zeros(56, 1024, dtype=torch.bfloat16, device="cuda")
        native.gemm(ctx, w, x, 56, out=out, splits=splits)
        outs.append(out)
    ctx.check()
    _close(outs[0], x.float() @ w.float().T)
    assert torch.equal(outs[0], outs[1]), "same split count must give bit-identical results"


@pytest.mark.parametrize("n_out,k,rows,splits", [(2048, 2048, 56, 1), (2048, 2048, 56, 3), (2048, 8192, 56, 16),
                                                  (1000, 1024, 42, 9), (640, 1024, 200, 4)])
def test_partial_epilogue(ctx, n_out, k, rows, splits):
    """PLM_EPI_PARTIAL writes each k-split's fp32 partial; summed in split order and rounded they equal the store
    epilogue at the same split count bit for bit (the cluster reduction adds the ranks in the same order)."""
    from plm import native

    w = _rand(n_out, k, scale=0.02, seed=11)
    x = _rand(rows, k, seed=12)
    part = torch.full((splits * rows, n_out), float("nan"), dtype=torch.float32, device="cuda")
    native.gemm(ctx, w, x, rows, out=part, epi=native.GemmEpilogue(kind=native.EPI_PARTIAL), splits=splits)
    ctx.check()
    slices = part.view(splits, rows, n_out)
    total = torch.zeros(rows, n_out, dtype=torch.float32, device="cuda")
    for s in range(splits):
        total = total + slices[s]
    _close(total, x.float() @ w.float().T)
    if splits <= 8 and rows <= 128:
        store = torch.zeros(rows, n_out, dtype=torch.bfloat16, device="cuda")
        native.gemm(ctx, w, x, rows, out=store, splits=splits)
        ctx.check()
        assert torch.equal(total.bfloat16(), store)


def test_partial_epilogue_needs_explicit_splits(ctx):
    from plm import native

    w, x = _rand(256, 256, seed=1), _rand(8, 256, seed=2)
    part = torch.zeros(64, 256, dtype=torch.float32, device="cuda")
    with pytest.raises(native.NativeError):
        native.gemm(ctx, w, x, 8, out=part, epi=native.GemmEpilogue(kind=native.EPI_PARTIAL))
    with pytest.raises(native.NativeError):
        native.gemm(ctx, w, x, 8, out=part, epi=native.GemmEpilogue(kind=native.EPI_PARTIAL), splits=17)


def test_padded_row_buffer(ctx):
    """Rows beyond `rows` in the operand buffer must not leak into the result (they are read by TMA, not stored)."""
    from plm import native

    w = _rand(512, 512, scale=0.02, seed=5)
    x = _rand(64, 512, seed=6)
    out = torch.zeros(64, 512, dtype=torch.bfloat16, device="cuda")
    native.gemm(ctx, w, x, 56, out=out)
    ctx.check()
    _close(out[:56], x[:56].float() @ w.float().T)
    assert torch.count_nonzero(out[56:]) == 0


@pytest.mark.parametrize("inter,hidden,rows", [(8192, 2048, 56), (2048, 512, 42), (256, 256, 20)])
def test_silu_mul_epilogue(ctx, inter, hidden, rows):
    from plm import native

    w = _rand(2 * inter, hidden, scale=0.02, seed=7)
    x = _rand(rows, hidden, seed=8)
    out = torch.zeros(rows, inter, dtype=torch.bfloat16, device="cuda")
    epi = native.GemmEpilogue(kind=native.EPI_SILU_MUL, gate_offset=inter)
    native.gemm(ctx, w, x, rows, out=out, epi=epi)
    ctx.check()
    y = (x.float() @ w.float().T).bfloat16().float()
    g, u = y[:, :inter], y[:, inter:]
    _close(out, torch.nn.functional.silu(g) * u)


def _cos_sin(max_pos, hd, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float) / hd))
    f = torch.arange(max_pos, dtype=torch.float)[:, None] * inv[None, :]
    return torch.cat([f.cos(), f.sin()], dim=-1).to(torch.bfloat16).cuda()


# (3, 1, 64): n_out = 320 leaves the last 128-feature tile half empty; page 24 is not a power of two
@pytest.mark.parametrize("heads,kv_heads,hd,rows,page", [(16, 16, 128, 56, 16), (8, 8, 64, 42, 16), (16, 4, 128, 56, 32),
                                                         (3, 1, 64, 20, 16), (8, 8, 64, 42, 24)])
def test_qkv_rope_kv_epilogue(ctx, heads, kv_heads, hd, rows, page):
    from plm import native

    hidden = heads * hd
    n_out = (heads + 2 * kv_heads) * hd
    w = _rand(n_out, hidden, scale=0.02, seed=9)
    x = _rand(rows, hidden, seed=10)
    max_pos, num_pages = 4096, 64
    cos_sin = _cos_sin(max_pos, hd)
    g = torch.Generator(device="cuda").manual_seed(11)
    positions = torch.randint(0, max_pos, (rows,), generator=g, device="cuda", dtype=torch.int32)
    slots = torch.randperm(num_pages * page, generator=g, device="cuda")[:rows].to(torch.int64)
    q_out = torch.zeros(rows, heads * hd, dtype=torch.bfloat16, device="cuda")
    k_cache = torch.zeros(num_pages, kv_heads, page, hd, dtype=torch.bfloat16, device="cuda")
    v_cache = torch.zeros_like(k_cache)
    epi = native.GemmEpilogue(kind=native.EPI_QKV_ROPE, q_out=q_out.data_ptr(), k_cache=k_cache.data_ptr(),
                              v_cache=v_cache.data_ptr(), positions=positions.data_ptr(), slots=slots.data_ptr(),
                              cos_sin=cos_sin.data_ptr(), num_heads=heads, num_kv_heads=kv_heads, head_dim=hd,
                              page_size=page, num_slots=num_pages * page, max_pos=max_pos)
    native.gemm(ctx, w, x, rows, epi=epi)
    ctx.check()

    y = (x.float() @ w.float().T).bfloat16().float()
    q = y[:, : heads * hd].view(rows, heads, hd)
    k = y[:, heads * hd: (heads + kv_heads) * hd].view(rows, kv_heads, hd)
    v = y[:, (heads + kv_heads) * hd:].view(rows, kv_heads, hd)
    cs = cos_sin[positions.long()].float()
    cos, sin = cs[:, None, : hd // 2], cs[:, None, hd // 2:]

    def rope(t):
        x1, x2 = t[..., : hd // 2], t[..., hd // 2:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    _close(q_out.view(rows, heads, hd), rope(q))
    page_of, within = slots // page, slots % page
    _close(k_cache[page_of, :, within, :], rope(k))
    _close(v_cache[page_of, :, within, :], v)
    # slots not written stay zero
    mask = torch.ones(num_pages * page, dtype=torch.bool, device="cuda")
    mask[slots] = False
    assert torch.count_nonzero(k_cache.permute(0, 2, 1, 3).reshape(num_pages * page, -1)[mask]) == 0
    assert torch.count_nonzero(v_cache.permute(0, 2, 1, 3).reshape(num_pages * page, -1)[mask]) == 0


@pytest.mark.parametrize("n_verify,rows", [(7, 56), (1, 56), (1, 1), (6, 42)])
def test_logits_epilogue(ctx, n_verify, rows):
    from plm import native

    vocab, hidden = 50257, 2048
    w = _rand(vocab, hidden, scale=0.02, seed=12)
    x = _rand(rows, hidden, seed=13)
    tiles = native.gemm_tiles(native.EPI_LOGITS, vocab)
    logits = torch.zeros(max(n_verify, 1), vocab, dtype=torch.float32, device="cuda")
    best_val = torch.zeros(tiles, rows, dtype=torch.float32, device="cuda")
    best_idx = torch.zeros(tiles, rows, dtype=torch.int32, device="cuda")
    epi = native.GemmEpilogue(kind=native.EPI_LOGITS, verify_logits=logits.data_ptr(), best_val=best_val.data_ptr(),
                              best_idx=best_idx.data_ptr(), n_verify=n_verify, vocab=vocab)
    native.gemm(ctx, w, x, rows, epi=epi)
    ctx.check()
    ref = (x.float() @ w.float().T)
    _close(logits[:n_verify], ref[:n_verify])
    # the stored logits are exactly model-dtype values
    assert torch.equal(logits[:n_verify], logits[:n_verify].bfloat16().float())
    if rows > n_verify:
        # reduce the per-tile partials in tile order: larger value, then smaller index
        vals, idxs = best_val[:, n_verify:], best_idx[:, n_verify:]
        top = vals.max(dim=0).values
        first = torch.where(vals == top[None, :], idxs, torch.full_like(idxs, 1 << 30)).min(dim=0).values
        # against the argmax of the kernel's own rounded values: recompute rows with the GEMM store path
        out = torch.zeros(rows, vocab, dtype=torch.bfloat16, device="cuda")
        native.gemm(ctx, w, x, rows, out=out)
        ctx.check()
        expect = out[n_verify:].float().argmax(dim=-1)
        mismatched = int((first.long() != expect).sum())
        assert mismatched == 0, f"{mismatched} proposal rows disagree with argmax of the stored logits"


def test_table_epilogue(ctx):
    from plm import native

    vocab, hidden, aux = 1000, 512, 512
    lm = _rand(vocab, hidden, scale=0.02, seed=14)
    vocab_aux = _rand(aux, hidden, seed=15)
    table = torch.zeros(vocab, aux, dtype=torch.bfloat16, device="cuda")
    for a0 in range(0, aux, 256):
        epi = native.GemmEpilogue(kind=native.EPI_TABLE, table=table.data_ptr(), aux=aux, a0=a0)
        native.gemm(ctx, lm, vocab_aux[a0:a0 + 256], 256, epi=epi)
    ctx.check()
    ref = -(vocab_aux.float() @ lm.float().T).T
    _close(table, ref)
