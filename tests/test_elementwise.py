"""plm_add_rmsnorm (vLLM's fused residual-add RMSNorm between the Llama sublayers) against a torch fp32 reference.

The new residual is the fp32 sum rounded to bf16, bit for bit. The normed row is bf16(bf16(v * rstd) * w) with rstd
from the unrounded fp32 sum of squares; the kernel's reduction order differs from torch's, so the normed row may
differ by one bf16 ulp of rounding.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


# 1032 and 4088 are multiples of 8 but not 16: clusters of 2 CTAs per row, 4088 with two quads on most threads
@pytest.mark.parametrize("rows,hidden,gather", [(56, 2048, -1), (7, 512, 3), (3, 2560, 0), (5, 4096, -1), (4, 1032, 1),
                                                (3, 4088, -1)])
def test_add_rmsnorm_matches_fp32(ctx, rows, hidden, gather):
    from plm import native

    g = torch.Generator(device="cuda").manual_seed(rows * hidden)
    x = torch.randn(rows, hidden, generator=g, device="cuda").bfloat16()
    res = (2 * torch.randn(rows, hidden, generator=g, device="cuda")).bfloat16()
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device="cuda")).bfloat16()
    eps = 1e-5
    v = x.float() + res.float()
    want_res = v.bfloat16()
    rstd = torch.rsqrt((v * v).mean(dim=1, keepdim=True) + eps)
    want = ((v * rstd).bfloat16().float() * w.float()).bfloat16()

    res_io = res.clone()
    normed = torch.empty_like(x)
    gathered = torch.zeros(hidden, dtype=torch.bfloat16, device="cuda")
    desc = native.AddRmsNormDesc(dtype=native.PLM_BF16, x=x.data_ptr(), residual=res_io.data_ptr(),
                                 normed=normed.data_ptr(), weight=w.data_ptr(), rows=rows, hidden=hidden, eps=eps,
                                 gather_row=gather, gathered=gathered.data_ptr() if gather >= 0 else None)
    native.add_rmsnorm(ctx, desc)
    ctx.check()
    assert torch.equal(res_io, want_res)
    ulp = torch.finfo(torch.bfloat16).eps * want.float().abs().clamp(min=2.0 ** -126) * 2
    assert ((normed.float() - want.float()).abs() <= ulp + 1e-30).all()
    if gather >= 0:
        assert torch.equal(gathered, normed[gather])


def test_add_rmsnorm_rejects_unsupported_width(ctx):
    from plm import native

    x = torch.zeros(2, 100, dtype=torch.bfloat16, device="cuda")
    desc = native.AddRmsNormDesc(dtype=native.PLM_BF16, x=x.data_ptr(), residual=x.data_ptr(), normed=x.data_ptr(),
                                 weight=x.data_ptr(), rows=2, hidden=100, eps=1e-5, gather_row=-1, gathered=None)
    with pytest.raises(native.NativeError):
        native.add_rmsnorm(ctx, desc)


@pytest.mark.parametrize("rows,hidden,splits", [(56, 2048, 16), (7, 512, 3), (3, 2560, 1), (5, 1032, 16), (2, 4088, 9)])
def test_add_rmsnorm_from_partials(ctx, rows, hidden, splits):
    """x given as fp32 k-split partials: summed in split order and rounded to bf16 first, then the same fused
    residual-add RMSNorm; equal bit for bit to the run with that bf16 x."""
    from plm import native

    g = torch.Generator(device="cuda").manual_seed(splits * hidden)
    part = torch.randn(splits, rows, hidden, generator=g, device="cuda")
    x = torch.zeros(rows, hidden, device="cuda")
    for s in range(splits):
        x = x + part[s]
    x = x.bfloat16()
    res = (2 * torch.randn(rows, hidden, generator=g, device="cuda")).bfloat16()
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device="cuda")).bfloat16()
    outs = []
    for use_partials in (False, True):
        res_io, normed = res.clone(), torch.empty_like(x)
        desc = native.AddRmsNormDesc(dtype=native.PLM_BF16, x=None if use_partials else x.data_ptr(),
                                     residual=res_io.data_ptr(), normed=normed.data_ptr(), weight=w.data_ptr(),
                                     rows=rows, hidden=hidden, eps=1e-5, gather_row=-1, gathered=None,
                                     partials=part.data_ptr() if use_partials else None,
                                     n_partials=splits if use_partials else 0,
                                     partial_stride=rows * hidden if use_partials else 0)
        native.add_rmsnorm(ctx, desc)
        ctx.check()
        outs.append((res_io, normed))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
