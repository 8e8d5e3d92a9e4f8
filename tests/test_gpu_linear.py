"""The tcgen05 projection GEMM (``lf_linear``) against torch's ``F.linear`` (cuBLAS).

Both accumulate in f32 and round once, in different orders, so outputs agree to
the bf16/f16 rounding of the result: the serving tolerance (2e-2 relative, max
error over max magnitude) with a far tighter norm-wise bound written below.  The
fused GELU is the f32 formula on the rounded projection, as ``F.gelu`` applies
it to the bf16 tensor.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from latefuse_b200 import _native as nat
from latefuse_b200.encoder_ops import ACT_GELU, linear, linear_accumulate

pytestmark = pytest.mark.gpu


def close(ours, ref):
    o, r = ours.float(), ref.float()
    err = (o - r).abs().max().item()
    assert err <= 2e-2 * r.abs().max().item(), err
    rel = ((o - r).norm() / r.norm().clamp_min(1e-12)).item()
    assert rel < 4e-3, rel


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(16401, 3072, 1024), (300, 1024, 1024), (129, 4096, 1024), (1000, 1024, 4096),
                                   (1, 256, 64), (128, 512, 192)])
def test_linear_matches_torch(cuda, dtype, m, n, k):
    g = torch.Generator(device="cpu").manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g).to(dtype).to(cuda)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(cuda)
    b = torch.randn(n, generator=g).to(dtype).to(cuda)
    close(linear(x, w, b), F.linear(x, w, b))
    close(linear(x, w, None), F.linear(x, w))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_gelu_matches_torch(cuda, dtype):
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(2000, 1024, generator=g).to(dtype).to(cuda)
    w = (torch.randn(4096, 1024, generator=g) * 1024 ** -0.5).to(dtype).to(cuda)
    b = torch.randn(4096, generator=g).to(dtype).to(cuda)
    ours = linear(x, w, b, act=ACT_GELU)
    close(ours, F.gelu(F.linear(x, w, b)))
    # the fused GELU is the formula applied to the kernel's own rounded projection, its
    # erf from a Chebyshev fit of erfc: within one ulp of the dtype, nearly always equal
    xf = linear(x, w, b).float()
    check_gelu(ours, xf, dtype)


def ulp_distance(a, b):
    """Distance in units in the last place between two 16-bit float tensors of one dtype
    (sign-magnitude bits mapped onto one integer line, so -0 and +0 coincide)."""
    def line(t):
        bits = t.contiguous().view(torch.int16).int()
        return torch.where(bits < 0, -(bits & 0x7FFF), bits)
    return (line(a) - line(b)).abs()


def check_gelu(got, v, dtype):
    """The epilogue's GELU against the formula v * 0.5 * (1 + erf(v / sqrt 2)) on the same
    rounded inputs v: within one ulp of the dtype, except where the formula itself is
    only as good as f32 cancellation makes it (for v below about -4, 1 + erf is a few
    units of 2^-24, so one ulp of erf moves the result by a factor): there within
    |v| * 2^-22 absolutely.  Elements that differ at all stay below 0.2% for bf16 and
    0.5% for f16 (three more mantissa bits: eight times the rounding boundaries)."""
    want = (v * 0.5 * (1.0 + torch.erf(v * 0.70710678118654752440))).to(dtype)
    dist = ulp_distance(got, want)
    near = (got.float() - want.float()).abs() <= v.abs() * 2.0 ** -22
    bad = (dist > 1) & ~near
    assert not bad.any(), (v[bad][:8].tolist(), got[bad][:8].float().tolist(), want[bad][:8].float().tolist())
    frac = (dist != 0).float().mean().item()
    assert frac < (2e-3 if dtype == torch.bfloat16 else 5e-3), frac


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_gelu_over_every_input_value(cuda, dtype):
    """Every finite 16-bit input through the GEMM epilogue's GELU (x one-hot in its
    first column, so the projection is the value itself): within one ulp of the
    formula everywhere, and the share that differs at all stays tiny."""
    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    vals = bits.view(dtype).float()
    vals = vals[torch.isfinite(vals)]
    m = vals.numel()
    x = torch.zeros(m, 64, dtype=dtype)
    x[:, 0] = vals.to(dtype)
    w = torch.zeros(256, 64, dtype=dtype)
    w[:, 0] = 1.0
    got = linear(x.to(cuda), w.to(cuda), None, act=ACT_GELU)[:, 0]
    check_gelu(got, vals.to(dtype).float().to(cuda), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(16401, 1024, 4096), (300, 1024, 1024), (1, 256, 64), (129, 512, 192)])
def test_linear_accumulate_matches_f32(cuda, dtype, m, n, k):
    """y += x W^T (+ b) in place, rounded once: against the f32 sum and torch's addmm_
    (beta = 1), with y a strided view whose other rows and columns stay untouched."""
    g = torch.Generator(device="cpu").manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, generator=g).to(dtype).to(cuda)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(cuda)
    b = torch.randn(n, generator=g).to(dtype).to(cuda)
    big = torch.randn(m + 3, n + 256, generator=g).to(dtype).to(cuda)
    before = big.clone()
    y = big[:m, :n]
    y0 = y.clone()
    assert linear_accumulate(x, w, y, b) is y
    close(y, y0.float() + x.float() @ w.float().T + b.float())
    assert torch.equal(big[m:], before[m:]) and torch.equal(big[:, n:], before[:, n:])
    y.copy_(y0)
    linear_accumulate(x, w, y)
    close(y, y0.clone().addmm_(x, w.t()))


def test_linear_accumulate_rejections(cuda):
    x = torch.randn(64, 1024, device=cuda, dtype=torch.bfloat16)
    w = torch.randn(1024, 1024, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="rows"):
        linear_accumulate(x, w, torch.zeros(63, 1024, device=cuda, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="float16"):
        linear_accumulate(x, w, torch.zeros(64, 1024, device=cuda, dtype=torch.float16))
    with pytest.raises(nat.NativeLibraryError, match="multiple of 256"):
        linear_accumulate(x, w[:1000], torch.zeros(64, 1000, device=cuda, dtype=torch.bfloat16))


def test_linear_strided_rows_and_rejections(cuda):
    x = torch.randn(500, 2048, device=cuda, dtype=torch.bfloat16)[:, :1024]   # row stride 2048
    w = torch.randn(768, 1024, device=cuda, dtype=torch.bfloat16) * 0.03
    out = torch.empty(500, 1024, device=cuda, dtype=torch.bfloat16)[:, :768]  # row stride 1024
    linear(x, w, None, out=out)
    close(out, F.linear(x, w))
    with pytest.raises(nat.NativeLibraryError, match="multiple of 256"):
        linear(x, torch.randn(100, 1024, device=cuda, dtype=torch.bfloat16), None)
    with pytest.raises(nat.NativeLibraryError, match="bf16 or f16"):
        linear(x.float(), w.float(), None)
    # an output that would need a copy to be seen as rows is refused, not written to a copy
    with pytest.raises(ValueError, match="viewable"):
        linear(x, w, None, out=torch.empty(768, 500, device=cuda, dtype=torch.bfloat16).t())
