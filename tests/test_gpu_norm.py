"""m3_rmsnorm against the reference RMSNorm formula (ops.py:94-102) evaluated in torch
on the same device, with and without the fused residual add (block.py:20-29).

Tolerances: fp32 rel 1e-5; bf16 / f16 outputs within one rounding step of the reference
(rel 1e-2), the residual sum bit-exact (it is one rounded add)."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref(x, w, eps, res=None):
    if res is not None:
        x = x + res
    xf = x.float()
    rms = xf.pow(2).mean(dim=-1, keepdim=True).add(eps).sqrt()
    return (xf / rms * w).to(x.dtype), x


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype,wdtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                          (torch.bfloat16, torch.float32), (torch.float16, torch.float32)])
@pytest.mark.parametrize("shape", [(256, 1536), (3, 7, 64), (5, 33), (1, 1)])
def test_rmsnorm_matches_formula(dtype, wdtype, shape):
    from mamba3_ssm.ops import rmsnorm
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(shape, device=DEV, generator=g).to(dtype)
    res = torch.randn(shape, device=DEV, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], device=DEV, generator=g)).to(wdtype)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    ref, _ = _ref(x, w, 1e-5)
    assert _rel(rmsnorm(x, w, 1e-5), ref) < tol
    ref, h_ref = _ref(x, w, 1e-5, res)
    h = torch.empty_like(x)
    out = rmsnorm(x, w, 1e-5, residual=res, residual_out=h)
    assert torch.equal(h, h_ref)
    assert _rel(out, ref) < tol
    # in place: the sum overwrites x
    x2 = x.clone()
    out2 = rmsnorm(x2, w, 1e-5, residual=res, residual_out=x2)
    assert torch.equal(x2, h_ref) and torch.equal(out2, out)


def test_rmsnorm_strided_views():
    """A last-dim slice of a wider row (the B / C slices of the in_proj output) and a
    view whose leading dims do not collapse."""
    from mamba3_ssm.ops import rmsnorm
    g = torch.Generator(device=DEV).manual_seed(4)
    base = torch.randn(4, 9, 300, device=DEV, generator=g)
    x = base[..., 100:164].unflatten(-1, (2, 32))      # (4, 9, 2, 32), leading dims not collapsible
    w = torch.rand(32, device=DEV, generator=g) + 0.5
    ref, _ = _ref(x, w, 1e-5)
    assert _rel(rmsnorm(x, w, 1e-5), ref) < 1e-5
    x2 = base[:, :, 10:74]                             # rows of stride 300
    ref, _ = _ref(x2, torch.ones(64, device=DEV), 1e-5)
    assert _rel(rmsnorm(x2, torch.ones(64, device=DEV), 1e-5), ref) < 1e-5


def test_rmsnorm_empty_and_errors():
    from mamba3_ssm.ops import rmsnorm
    w = torch.ones(16, device=DEV)
    assert rmsnorm(torch.empty(0, 16, device=DEV), w, 1e-5).shape == (0, 16)
    with pytest.raises(RuntimeError, match="weight"):
        rmsnorm(torch.randn(4, 16, device=DEV), torch.ones(15, device=DEV), 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(256, 50000), (3, 7), (2, 5, 1003), (1, 64)])
def test_argmax_rows_matches_torch(dtype, shape):
    """m3_argmax_rows == torch.argmax(-1): first index of the maximum, ties and NaN rows
    included, vector and element-wise paths."""
    from mamba3_ssm.ops import argmax_rows
    g = torch.Generator(device="cpu").manual_seed(sum(shape))
    x = torch.randn(shape, generator=g).to(dtype)
    flat = x.reshape(-1, shape[-1])
    flat[0, :] = 1.0                       # all ties: index 0
    if flat.shape[0] > 1:
        flat[1, shape[-1] // 2] = float("nan")  # NaN counts as the maximum
    if flat.shape[0] > 2 and shape[-1] > 3:
        flat[2, 1] = flat[2, 3] = 100.0    # repeated maximum: the first
    x = x.to(DEV)
    got = argmax_rows(x)
    assert got.dtype == torch.int64 and got.shape == x.shape[:-1]
    assert torch.equal(got, x.argmax(-1))
    out = torch.empty(x.shape[:-1], dtype=torch.int64, device=DEV)
    argmax_rows(x, out=out)
    assert torch.equal(out, x.argmax(-1))
