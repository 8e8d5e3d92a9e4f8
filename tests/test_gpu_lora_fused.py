"""The one-launch LoRA delta (lf_lora_apply's fused kernel) against the shrink + expand
launches and the oracle.

Both paths accumulate u over the whole hidden dimension with the same MMA sequence
and round at the same points, so the one-launch kernel must give the same bits as the
two launches; the oracle bound (bf16/f16: 2e-2 relative on the delta, as stated for
the serving path) is checked as well.
"""

from __future__ import annotations

import pytest
import torch

from latefuse_b200 import _native as nat
from latefuse_b200.lora import SegmentTable, lora_apply, workspace_bytes
from oracle.lora import segmented_apply
from tests.test_gpu_lora_kernels import check, make_cache

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _options():
    nat.set_option(nat.LF_OPT_REQUIRE_TC, 1)
    nat.set_option(nat.LF_OPT_FUSED_APPLY, 1)
    nat.set_option(nat.LF_OPT_FUSED_SPLIT, 0)
    yield
    nat.set_option(nat.LF_OPT_REQUIRE_TC, 0)
    nat.set_option(nat.LF_OPT_FUSED_APPLY, 1)
    nat.set_option(nat.LF_OPT_FUSED_SPLIT, 0)


def apply(x, y, fc, st, mods, offs, fused=True, split=0):
    ws = torch.empty(workspace_bytes(x.dtype, x.shape[0], fc.rank, len(mods)), dtype=torch.uint8, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    out = y.clone()
    # several modules take the one-launch kernel only when asked for (2)
    nat.set_option(nat.LF_OPT_FUSED_APPLY, (1 if len(mods) == 1 else 2) if fused else 0)
    nat.set_option(nat.LF_OPT_FUSED_SPLIT, split)
    n0 = nat.launch_count()
    lora_apply(x, out, fc, st, mods, offs, ws, status)
    torch.cuda.synchronize()
    launches = nat.launch_count() - n0
    nat.set_option(nat.LF_OPT_FUSED_APPLY, 1)
    nat.set_option(nat.LF_OPT_FUSED_SPLIT, 0)
    return out, status.item(), launches


def short_segments(n, gap_max, n_slots, g):
    lengths = torch.randint(1, 40, (n,), generator=g).tolist()
    gaps = torch.randint(0, gap_max, (n,), generator=g).tolist()
    starts, t = [], 0
    for ln, gap in zip(lengths, gaps):
        t += gap
        starts.append(t)
        t += ln
    slots = torch.randint(0, n_slots, (n,), generator=g).tolist()
    return starts, lengths, slots, t


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n_mod,R", [(1, 8), (1, 16), (1, 64), (3, 16), (3, 32), (4, 16), (3, 64), (4, 64), (2, 8)])
def test_fused_equals_two_launches_many_segments(cuda, dtype, n_mod, R):
    """Tiles holding up to ~15 short segments with gaps (several rounds per record for
    every rank and module count), a partial last tile, every column chunking: the one
    launch gives the two launches' bits.  Several modules run the kernel only under
    LF_OPT_FUSED_APPLY = 2; by default they take the two launches."""
    H, n_slots = 512, 11
    g = torch.Generator().manual_seed(31 * n_mod + R)
    starts, lengths, slots, t = short_segments(40, 6, n_slots, g)
    T = t + 37
    fc, a_of, b_of = make_cache(n_slots, n_mod, H, R, dtype, cuda, seed=R + n_mod)
    x = torch.randn(T, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(T, n_mod * H, generator=g).to(dtype).to(cuda)
    mods, offs = list(range(n_mod)), [m * H for m in range(n_mod)]
    st = SegmentTable(starts, lengths, slots, T, cuda)
    assert st.n_multi > 0
    two, s2, l2 = apply(x, y, fc, st, mods, offs, fused=False)
    assert s2 == 0 and l2 == 2
    # three or four modules of rank 64 do not fit the one-launch kernel's rings and take
    # the two launches even under LF_OPT_FUSED_APPLY = 2
    fits = n_mod * R < 192
    for split in (0, 1, 2, 4):
        one, s1, l1 = apply(x, y, fc, st, mods, offs, split=split)
        assert s1 == 0, nat.decode_status(s1)
        assert l1 == (1 if fits else 2)
        assert torch.equal(one, two), f"split {split}"
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, list(zip(starts, lengths, slots)), col_offsets=offs,
                          modules=mods)
    check(two.cpu(), ref, y.cpu(), dtype)


@pytest.mark.parametrize("R,n_slots", [(8, 10_000), (16, 10_000), (64, 2_500)])
def test_fused_isolated_op_shape(cuda, R, n_slots):
    """The isolated op: X (64, 256, 1024), 10,000 cached tenants (2,500 at rank 64, to
    keep the host-side copy small), one tenant per row drawn Zipf(1.1); fused and
    two-launch paths equal, and the delta matches the oracle on a few rows."""
    dtype, B, S, H = torch.bfloat16, 64, 256, 1024
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=5, std=0.02)
    gen = torch.Generator().manual_seed(R)
    x = torch.randn(B * S, H, generator=gen).to(dtype).to(cuda)
    y = torch.randn(B * S, H, generator=gen).to(dtype).to(cuda)
    w = 1.0 / torch.arange(1, n_slots + 1, dtype=torch.float64) ** 1.1
    tenant = torch.multinomial(w, B, replacement=True, generator=gen)
    order = torch.argsort(tenant, stable=True)  # rows sorted by tenant: one segment per run
    x = x.view(B, S, H)[order.to(cuda)].reshape(B * S, H)
    t_sorted = tenant[order].tolist()
    segs, b = [], 0
    while b < B:
        e = b
        while e < B and t_sorted[e] == t_sorted[b]:
            e += 1
        segs.append((b * S, (e - b) * S, t_sorted[b]))
        b = e
    st = SegmentTable([s for s, _, _ in segs], [n for _, n, _ in segs], [k for _, _, k in segs], B * S, cuda)
    two, s2, _ = apply(x, y, fc, st, [0], [0], fused=False)
    one, s1, l1 = apply(x, y, fc, st, [0], [0])
    assert s1 == 0 and s2 == 0 and l1 == 1
    assert torch.equal(one, two)
    rows = torch.cat([torch.arange(s, s + 200) for s, _, _ in segs[:3]])
    local = [(200 * i, 200, k) for i, (_, _, k) in enumerate(segs[:3])]
    ref = segmented_apply(x.cpu()[rows], y.cpu()[rows], a_of, b_of, local)
    check(one.cpu()[rows], ref, y.cpu()[rows], dtype)


def test_fused_column_slices_of_a_wider_output(cuda):
    """Modules writing column slices of a wider y (q/k/v of one (T, 4H) buffer, module
    order not the column order) leave every other column untouched."""
    dtype, H, R, n_slots = torch.bfloat16, 256, 16, 5
    g = torch.Generator().manual_seed(9)
    starts, lengths, slots, t = short_segments(12, 30, n_slots, g)
    T = t + 3
    fc, a_of, b_of = make_cache(n_slots, 3, H, R, dtype, cuda, seed=3)
    x = torch.randn(T, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(T, 4 * H, generator=g).to(dtype).to(cuda)
    mods, offs = [2, 0, 1], [H, 3 * H, 0]
    st = SegmentTable(starts, lengths, slots, T, cuda)
    two, _, _ = apply(x, y, fc, st, mods, offs, fused=False)
    one, s1, _ = apply(x, y, fc, st, mods, offs)
    assert s1 == 0 and torch.equal(one, two)
    assert torch.equal(one[:, 2 * H:3 * H], y[:, 2 * H:3 * H])
    # by default (LF_OPT_FUSED_APPLY = 1) several modules take the two launches
    ws = torch.empty(workspace_bytes(dtype, T, R, 3), dtype=torch.uint8, device=cuda)
    out = y.clone()
    n0 = nat.launch_count()
    lora_apply(x, out, fc, st, mods, offs, ws)
    torch.cuda.synchronize()
    assert nat.launch_count() - n0 == 2 and torch.equal(out, two)
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, list(zip(starts, lengths, slots)), col_offsets=offs,
                          modules=mods)
    check(one.cpu(), ref, y.cpu(), dtype)


def test_fused_rows_outside_segments_keep_their_values(cuda):
    """Rows in no segment (padding inside a record's tile) keep their values: negative
    zeros bit for bit, NaNs as NaNs (a row that shares its 32-row box with segment rows
    gets -0 added, which may return NaN with another payload)."""
    dtype, H, R, n_slots = torch.bfloat16, 256, 16, 3
    T = 300
    fc, _, _ = make_cache(n_slots, 1, H, R, dtype, cuda, seed=4)
    x = torch.randn(T, H, device=cuda).to(dtype)
    y = torch.randn(T, H, device=cuda).to(dtype)
    y[10:20] = -0.0
    y[150:160, 7] = float("nan")
    st = SegmentTable([0, 40, 200], [10, 100, 50], [2, 0, 1], T, cuda)
    one, s1, _ = apply(x, y, fc, st, [0], [0])
    assert s1 == 0
    keep = torch.ones(T, dtype=torch.bool, device=cuda)
    for s0, n in ((0, 10), (40, 100), (200, 50)):
        keep[s0:s0 + n] = False
    nan = torch.isnan(y)
    assert torch.equal(torch.isnan(one), nan)
    assert torch.equal(one[keep & ~nan.any(1)].view(torch.int16), y[keep & ~nan.any(1)].view(torch.int16))
    assert not torch.equal(one[~keep], y[~keep])


def test_fused_bad_slot_is_reported_without_fault(cuda):
    """A segment naming a slot outside the cache: its rows get no delta, the status
    word says so, the other segments are served."""
    dtype, H, R, n_slots = torch.bfloat16, 256, 16, 4
    T = 256
    fc, _, _ = make_cache(n_slots, 1, H, R, dtype, cuda, seed=6)
    x = torch.randn(T, H, device=cuda).to(dtype)
    y = torch.randn(T, H, device=cuda).to(dtype)
    st = SegmentTable([0, 100], [100, 156], [1, 7], T, cuda)
    one, s1, _ = apply(x, y, fc, st, [0], [0])
    assert s1 & 1, nat.decode_status(s1)  # LF_STATUS_BAD_SLOT
    assert torch.equal(one[100:], y[100:])
    assert not torch.equal(one[:100], y[:100])
