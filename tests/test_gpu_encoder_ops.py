"""The encoder's native elementwise kernels against torch's own ops on the same
GPU: residual add + LayerNorm (f32 1e-5; bf16/f16 within one or two output
ulps, the only difference being the order of the f32 row sums) and the exact
GELU."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from latefuse_b200 import _native as nat
from latefuse_b200.encoder_ops import add_layernorm, embed_layernorm, gelu

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (2e-2, 1.6e-2), torch.float16: (4e-3, 2e-3)}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H", [64, 768, 1024, 2560, 4096])
@pytest.mark.parametrize("residual", [True, False])
def test_add_layernorm_matches_torch(cuda, dtype, H, residual):
    g = torch.Generator(device=cuda).manual_seed(H)
    rows = 1000
    a = (torch.randn(rows, H, device=cuda, generator=g) * 3 + 1).to(dtype)
    b = torch.randn(rows, H, device=cuda, generator=g).to(dtype) if residual else None
    w = (1 + 0.1 * torch.randn(H, device=cuda, generator=g)).to(dtype)
    bias = (0.1 * torch.randn(H, device=cuda, generator=g)).to(dtype)
    ours = add_layernorm(a, b, w, bias, 1e-5)
    ref = F.layer_norm(a + b if residual else a, (H,), w, bias, 1e-5)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(ours, ref, atol=atol, rtol=rtol)
    if dtype != torch.float32:  # nearly every element is bit-identical
        assert (ours != ref).float().mean().item() < 0.02


def test_add_layernorm_in_place_and_strided(cuda):
    dtype, H = torch.bfloat16, 1024
    base = torch.randn(300, 2 * H, device=cuda).to(dtype)
    a = base[:, :H]  # row stride 2H
    b = torch.randn(300, H, device=cuda).to(dtype)
    w = torch.ones(H, device=cuda, dtype=dtype)
    z = torch.zeros(H, device=cuda, dtype=dtype)
    ref = F.layer_norm(a + b, (H,), w, z, 1e-12)
    out = b.clone()
    add_layernorm(a, out, w, z, 1e-12, out=out)  # out aliases the residual
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=1.6e-2)


def test_add_layernorm_rejects_bad_shapes(cuda):
    a = torch.randn(4, 12, device=cuda)
    with pytest.raises(nat.NativeLibraryError, match="multiple of 8"):
        add_layernorm(a, None, torch.ones(12, device=cuda), torch.zeros(12, device=cuda), 1e-5)
    a = torch.randn(4, 8192, device=cuda)
    with pytest.raises(nat.NativeLibraryError, match="4096"):
        add_layernorm(a, None, torch.ones(8192, device=cuda), torch.zeros(8192, device=cuda), 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_gelu_matches_torch(cuda, dtype):
    x = (torch.randn(16401, 4096, device=cuda) * 4).to(dtype)
    ours = gelu(x)
    ref = F.gelu(x)
    if dtype == torch.float32:
        torch.testing.assert_close(ours, ref, atol=1e-6, rtol=1e-6)
    else:
        torch.testing.assert_close(ours, ref, atol=0, rtol=8e-3)
        assert (ours != ref).float().mean().item() < 1e-3
    y = x.clone()
    gelu(y, out=y)
    assert torch.equal(y, ours)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gelu_every_2byte_input_matches_the_f32_formula(cuda, dtype):
    """The table path covers every bit pattern: each must equal the f32 formula rounded once."""
    bits = torch.arange(-32768, 32768, dtype=torch.int32, device=cuda).to(torch.int16)
    x = bits.view(dtype)
    ours = gelu(x)
    xf = x.float()
    ref = (xf * 0.5 * (1.0 + torch.erf(xf * 0.70710678118654752440))).to(dtype)
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(ours), nan)
    assert torch.equal(ours.view(torch.int16)[~nan], ref.view(torch.int16)[~nan])
    # odd lengths and offsets of whole 16-byte vectors
    for n in (8, 8 * 1023, 8 * 1025 + 8):
        torch.testing.assert_close(gelu(x[:n].clone()), ours[:n], atol=0, rtol=0, equal_nan=True)


def test_gelu_under_stream_capture(cuda):
    x = (torch.randn(4096, 1024, device=cuda) * 3).to(torch.bfloat16)
    ref = gelu(x)
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            gelu(x, out=out)
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_layernorm_with_row_vector_matches_torch(cuda, dtype):
    """LayerNorm(round(a + v)) for one row v added to every row (a projection bias)."""
    a = torch.randn(3000, 1024, device=cuda).to(dtype)
    v = torch.randn(1024, device=cuda).to(dtype)
    w = (torch.rand(1024, device=cuda) + 0.5).to(dtype)
    bias = torch.randn(1024, device=cuda).to(dtype)
    ours = add_layernorm(a, None, w, bias, 1e-5, vec=v)
    ref = F.layer_norm((a + v).float(), (1024,), w.float(), bias.float(), 1e-5).to(dtype)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(ours, ref, atol=tol, rtol=tol)
    assert (ours.float() - ref.float()).abs().max().item() <= (1e-5 if dtype == torch.float32 else 2 ** -6 * 8)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H", [256, 1024, 2560])
def test_embed_layernorm_is_the_gathers_adds_and_layernorm(cuda, dtype, H):
    """One launch for the packed forward's embeddings: the same bits as this library's
    add+LayerNorm on torch's own gathers and first add (the rounding points of the
    encoder's embeddings), token types given or all zero; an index outside its table
    is reported in the status word and reads row 0."""
    g = torch.Generator(device=cuda).manual_seed(H)
    V, P, n = 5000, 600, 3000
    word = torch.randn(V, H, device=cuda, generator=g).to(dtype)
    pos = torch.randn(P, H, device=cuda, generator=g).to(dtype)
    typ = torch.randn(2, H, device=cuda, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(H, device=cuda, generator=g)).to(dtype)
    b = (0.1 * torch.randn(H, device=cuda, generator=g)).to(dtype)
    ids = torch.randint(0, V, (n,), device=cuda, generator=g, dtype=torch.int32)
    positions = torch.randint(0, P, (n,), device=cuda, generator=g, dtype=torch.int32)
    types = torch.randint(0, 2, (n,), device=cuda, generator=g, dtype=torch.int32)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for tt in (types, None):
        ours = embed_layernorm(ids, positions, tt, word, pos, typ, w, b, 1e-5, status=status)
        x = word[ids.long()] + typ[tt.long() if tt is not None else torch.zeros_like(ids).long()]
        want = add_layernorm(x, pos[positions.long()], w, b, 1e-5)
        assert torch.equal(ours, want)
        ref = F.layer_norm((x.float() + pos[positions.long()].float()).to(dtype).float(), (H,), w.float(), b.float(),
                           1e-5)
        lo, hi = TOL[dtype]
        assert (ours.float() - ref).abs().max().item() <= lo
    torch.cuda.synchronize()
    assert status.item() == 0
    bad = ids.clone()
    bad[7] = V + 3
    ours = embed_layernorm(bad, positions, types, word, pos, typ, w, b, 1e-5, status=status)
    torch.cuda.synchronize()
    assert status.item() == nat.LF_STATUS_BAD_SLOT
    assert torch.isfinite(ours.float()).all()
