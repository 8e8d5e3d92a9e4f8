"""``lf_lora_apply_into``: the delta written into a fresh output (with an optional
residual and bias) for a beta = 1 GEMM to accumulate onto.

Its definition is ``y = round(round(r + bias) + round(delta))``, which is
``lf_lora_apply`` run in place on ``y0 = round(r + bias)``: the two must agree
bit for bit, on every token (the output starts as NaN, so a row left unwritten
fails).  The fused projection ``y.addmm_(x, W.t())`` is checked
against the reference's order (biased projection, then the delta, then the
residual) within the bf16 tolerance of the serving path (2e-2 relative).
"""

from __future__ import annotations

import pytest
import torch

from latefuse_b200 import _native as nat
from latefuse_b200.lora import FactorCache, SegmentTable, lora_apply, lora_apply_into, workspace_bytes

pytestmark = pytest.mark.gpu


def make_cache(n_slots, n_mod, H, R, dtype, dev, seed=0, std=0.05):
    """Cache in the store's slot layout with one layer: [slot][module][A (H,R) | B (R,H)]."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    buf = (torch.randn(n_slots, n_mod, 2, H * R, generator=g) * std).to(dtype).to(dev)
    return FactorCache(a=buf, b=buf, a_offset=0, b_offset=H * R, a_slot_stride=buf.stride(0),
                       b_slot_stride=buf.stride(0), a_module_stride=buf.stride(1), b_module_stride=buf.stride(1),
                       n_slots=n_slots, hidden=H, rank=R)


def packed_segments(n_rows, n_slots, seed, max_len=300):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (n_rows,), generator=g).tolist()
    slots = sorted(torch.randint(0, n_slots, (n_rows,), generator=g).tolist())
    starts, lengths, sl = [], [], []
    pos = 0
    for n, s in zip(lens, slots):
        if sl and sl[-1] == s:
            lengths[-1] += n
        else:
            starts.append(pos)
            lengths.append(n)
            sl.append(s)
        pos += n
    return starts, lengths, sl, pos


def run_into(x, y_shape, fc, st, modules, offs, residual, bias):
    dev = x.device
    ws = torch.empty(workspace_bytes(x.dtype, x.shape[0], fc.rank, len(modules)), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    y = torch.full(y_shape, float("nan"), dtype=x.dtype, device=dev)
    lora_apply_into(x, y, fc, st, modules, offs, ws, status, residual=residual, bias=bias)
    torch.cuda.synchronize()
    assert status.item() == 0, nat.decode_status(status.item())
    return y


def run_ref(x, y0, fc, st, modules, offs):
    ws = torch.empty(workspace_bytes(x.dtype, x.shape[0], fc.rank, len(modules)), dtype=torch.uint8, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    y = y0.clone()
    lora_apply(x, y, fc, st, modules, offs, ws, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    return y


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("R", [8, 16, 64])
@pytest.mark.parametrize("with_r,with_b", [(False, True), (True, True), (True, False), (False, False)])
def test_tc_into_matches_apply_on_r_plus_bias(cuda, dtype, R, with_r, with_b):
    H, n_slots = 256, 9
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(23, n_slots, seed=R + 7 * with_r + 3 * with_b)
    fc = make_cache(n_slots, 3, H, R, dtype, dev, seed=R)
    st = SegmentTable(starts, lengths, slots, T, dev)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(T, H, generator=g).to(dtype).to(dev)
    for modules, offs, W in [([0, 1, 2], [0, H, 2 * H], 3 * H), ([1], [0], H)]:
        r = torch.randn(T, W, generator=g).to(dtype).to(dev) if with_r else None
        b = torch.randn(W, generator=g).to(dtype).to(dev) if with_b else None
        y0 = torch.zeros(T, W, dtype=dtype, device=dev)
        if r is not None:
            y0 += r
        if b is not None:
            y0 += b
        ours = run_into(x, (T, W), fc, st, modules, offs, r, b)
        ref = run_ref(x, y0, fc, st, modules, offs)
        assert not torch.isnan(ours).any()
        assert torch.equal(ours, ref), (ours.float() - ref.float()).abs().max().item()


def test_tc_into_then_gemm_matches_reference_order(cuda):
    """y.addmm_(x, W^T) after the into call against round(round(xW^T + b) + delta) + r."""
    H, R, n_slots, dtype = 1024, 16, 12, torch.bfloat16
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(40, n_slots, seed=5, max_len=512)
    fc = make_cache(n_slots, 1, H, R, dtype, dev, seed=3)
    st = SegmentTable(starts, lengths, slots, T, dev)
    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(T, H, generator=g).to(dtype).to(dev)
    W = (torch.randn(H, H, generator=g) * 0.03).to(dtype).to(dev)
    b = torch.randn(H, generator=g).to(dtype).to(dev)
    r = torch.randn(T, H, generator=g).to(dtype).to(dev)
    fused = run_into(x, (T, H), fc, st, [0], [0], r, b)
    fused.addmm_(x, W.t())
    ref = run_ref(x, torch.nn.functional.linear(x, W, b), fc, st, [0], [0]) + r
    torch.cuda.synchronize()
    err = (fused.float() - ref.float()).abs().max().item()
    assert err <= 2e-2 * ref.float().abs().max().item(), err
    # three bf16 roundings on each side, at different points: a few 1e-3 in norm
    rel = ((fused.float() - ref.float()).norm() / ref.float().norm()).item()
    assert rel < 1e-2, rel


def test_into_rejects_uncovered_tokens_and_aliasing(cuda):
    H, R, dtype = 256, 16, torch.bfloat16
    dev = torch.device("cuda")
    fc = make_cache(2, 1, H, R, dtype, dev)
    x = torch.randn(300, H, dtype=dtype, device=dev)
    ws = torch.empty(workspace_bytes(dtype, 300, R, 1), dtype=torch.uint8, device=dev)
    partial = SegmentTable([0], [200], [0], 300, dev)
    with pytest.raises(ValueError):
        lora_apply_into(x, torch.empty(300, H, dtype=dtype, device=dev), fc, partial, [0], [0], ws)
    full = SegmentTable([0], [300], [0], 300, dev)
    y = torch.empty(300, H, dtype=dtype, device=dev)
    with pytest.raises(nat.NativeLibraryError):
        lora_apply_into(x, y, fc, full, [0], [0], ws, residual=y)
