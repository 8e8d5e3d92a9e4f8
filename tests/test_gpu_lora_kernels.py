"""Parity of the native LoRA kernels (tcgen05 and CUDA-core paths) with the oracle.

Tolerances: f32 1e-5 absolute; bf16/f16 2e-2 relative (max-abs error over the
max-abs of the oracle's delta), as stated for the serving path.  The oracle
reproduces the reference's rounding points (shrink output and delta stored in
the model dtype, add in the model dtype).
"""

from __future__ import annotations

import pytest
import torch

from latefuse_b200 import _native as nat
from latefuse_b200.lora import FactorCache, SegmentTable, lora_apply, lora_expand, lora_shrink, workspace_bytes
from oracle.lora import segmented_apply

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def make_cache(n_slots, n_mod, H, R, dtype, dev, seed=0, std=0.05):
    """Cache in the store's slot layout with one layer: [slot][module][A (H,R) | B (R,H)]."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    buf = (torch.randn(n_slots, n_mod, 2, H * R, generator=g) * std).to(dtype).to(dev)
    fc = FactorCache(a=buf, b=buf, a_offset=0, b_offset=H * R, a_slot_stride=buf.stride(0),
                     b_slot_stride=buf.stride(0), a_module_stride=buf.stride(1), b_module_stride=buf.stride(1),
                     n_slots=n_slots, hidden=H, rank=R)
    cpu = buf.cpu()

    def a_of(slot, m):
        return cpu[slot, m, 0].view(H, R)

    def b_of(slot, m):
        return cpu[slot, m, 1].view(R, H)

    return fc, a_of, b_of


def segments_padded(B, S, n_slots, seed, lengths=None):
    g = torch.Generator().manual_seed(seed)
    slots = torch.randint(0, n_slots, (B,), generator=g).tolist()
    lens = [S] * B if lengths is None else lengths
    return [(b * S, lens[b], slots[b]) for b in range(B)]


def run_apply(x, y, fc, segs, modules, offs, records=True):
    dev = x.device
    st = SegmentTable([s for s, _, _ in segs], [l for _, l, _ in segs], [k for _, _, k in segs], x.shape[0], dev,
                      records=records)
    ws = torch.empty(workspace_bytes(x.dtype, x.shape[0], fc.rank, len(modules)), dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = y.clone()
    lora_apply(x, out, fc, st, modules, offs, ws, status)
    torch.cuda.synchronize()
    assert status.item() == 0, nat.decode_status(status.item())
    return out


def check(ours, ref, base, dtype):
    d_ours = ours.float() - base.float()
    d_ref = ref.float() - base.float()
    scale = max(d_ref.abs().max().item(), 1e-6)
    err = (ours.float() - ref.float()).abs().max().item()
    if dtype == torch.float32:
        assert err <= TOL[dtype], f"max abs err {err}"
    else:
        # the final add rounds to the output dtype: allow one output ulp on top of the relative bound
        ulp = base.float().abs().max().item() * 2 ** -7
        assert err <= TOL[dtype] * scale + ulp, f"max abs err {err} vs delta scale {scale}"
        rel = (d_ours - d_ref).norm() / d_ref.norm().clamp_min(1e-12)
        assert rel.item() <= TOL[dtype], f"relative delta error {rel.item()}"


@pytest.fixture(autouse=True)
def _reset_options(request):
    # tests named test_tc_* must run on the tcgen05 kernels: falling back is an error
    nat.set_option(nat.LF_OPT_REQUIRE_TC, 1 if request.node.name.startswith("test_tc_") else 0)
    nat.set_option(nat.LF_OPT_FORCE_SIMT, 0)
    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 0)
    nat.set_option(nat.LF_OPT_PERSISTENT, 1)
    yield
    nat.set_option(nat.LF_OPT_PERSISTENT, 1)
    nat.set_option(nat.LF_OPT_REQUIRE_TC, 0)
    nat.set_option(nat.LF_OPT_FORCE_SIMT, 0)
    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_tc_padded_one_segment_per_tile(cuda, dtype, R):
    B, S, H, n_slots = 4, 128, 256, 7
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=R)
    x = torch.randn(B * S, H, generator=torch.Generator().manual_seed(1)).to(dtype).to(cuda)
    y = torch.randn(B * S, H, generator=torch.Generator().manual_seed(2)).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=3)
    ours = run_apply(x, y, fc, segs, [0], [0]).cpu()
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs)
    check(ours, ref, y.cpu(), dtype)


@pytest.mark.parametrize("R", [8, 16, 64])
def test_tc_delta_only_precision(cuda, R):
    """accumulate=0 isolates the delta: bf16 relative error well inside 2e-2."""
    dtype = torch.bfloat16
    T, H, n_slots = 384, 512, 5
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=11)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(4)).to(dtype).to(cuda)
    segs = [(0, 128, 1), (128, 200, 4), (328, 56, 0)]
    st = SegmentTable([s for s, _, _ in segs], [l for _, l, _ in segs], [k for _, _, k in segs], T, cuda)
    u = torch.empty(1, T, R, dtype=dtype, device=cuda)
    y = torch.full((T, H), 7.0, dtype=dtype, device=cuda)
    lora_shrink(x, u, fc, st, [0])
    lora_expand(u, y, fc, st, [0], [0], accumulate=False)
    torch.cuda.synchronize()
    ref = segmented_apply(x.cpu(), torch.zeros(T, H, dtype=dtype), a_of, b_of, segs, accumulate=False)
    rel = (y.cpu().float() - ref.float()).norm() / ref.float().norm()
    assert rel.item() < 5e-3, rel.item()


@pytest.mark.parametrize("H", [64, 192, 320])
def test_tc_hidden_not_multiple_of_128(cuda, H):
    dtype = torch.bfloat16
    B, S, R, n_slots = 3, 128, 16, 4
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=H)
    x = torch.randn(B * S, H, generator=torch.Generator().manual_seed(5)).to(dtype).to(cuda)
    y = torch.randn(B * S, H, generator=torch.Generator().manual_seed(6)).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=7)
    ours = run_apply(x, y, fc, segs, [0], [0]).cpu()
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs)
    check(ours, ref, y.cpu(), dtype)


@pytest.mark.parametrize("S", [16, 100, 200, 513])
def test_tc_ragged_segments_cross_tiles(cuda, S):
    """Sequences shorter/longer than a 128-token tile, a ragged last tile, skipped padding."""
    dtype = torch.bfloat16
    B, H, R, n_slots = 5, 256, 16, 9
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=S)
    g = torch.Generator().manual_seed(S)
    lengths = torch.randint(1, S + 1, (B,), generator=g).tolist()
    x = torch.randn(B * S, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(B * S, H, generator=g).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=S + 1, lengths=lengths)
    ours = run_apply(x, y, fc, segs, [0], [0]).cpu()
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs)
    check(ours, ref, y.cpu(), dtype)
    # rows outside every segment are bit-identical to the input
    covered = torch.zeros(B * S, dtype=torch.bool)
    for s, l, _ in segs:
        covered[s : s + l] = True
    assert torch.equal(ours[~covered], y.cpu()[~covered])


@pytest.mark.parametrize("modules,offs", [([0, 1, 2], [0, 1, 2]), ([0, 2], [0, 2]), ([1], [2])])
def test_tc_fused_qkv_modules(cuda, modules, offs):
    dtype = torch.bfloat16
    B, S, H, R, n_slots = 2, 256, 256, 16, 6
    fc, a_of, b_of = make_cache(n_slots, 3, H, R, dtype, cuda, seed=21)
    x = torch.randn(B * S, H, generator=torch.Generator().manual_seed(8)).to(dtype).to(cuda)
    y = torch.randn(B * S, 3 * H, generator=torch.Generator().manual_seed(9)).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=10)
    col = [o * H for o in offs]
    ours = run_apply(x, y, fc, segs, modules, col).cpu()
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs, col_offsets=col, modules=modules)
    check(ours, ref, y.cpu(), dtype)
    untouched = [j for j in range(3) if j not in offs]
    for j in untouched:
        assert torch.equal(ours[:, j * H : (j + 1) * H], y.cpu()[:, j * H : (j + 1) * H])


@pytest.mark.parametrize("csize", [1, 2, 4])
def test_tc_cluster_split_is_deterministic_and_equal(cuda, csize):
    dtype = torch.bfloat16
    B, S, H, R, n_slots = 2, 128, 256, 16, 3
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=31)
    x = torch.randn(B * S, H, generator=torch.Generator().manual_seed(12)).to(dtype).to(cuda)
    y = torch.randn(B * S, H, generator=torch.Generator().manual_seed(13)).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=14)
    nat.set_option(nat.LF_OPT_PERSISTENT, 0)  # the split-K kernel, not the persistent one
    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, csize)
    a = run_apply(x, y, fc, segs, [0], [0])
    b = run_apply(x, y, fc, segs, [0], [0])
    assert torch.equal(a, b)
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs)
    check(a.cpu(), ref, y.cpu(), dtype)


def test_tc_matches_simt(cuda):
    dtype = torch.bfloat16
    B, S, H, R, n_slots = 3, 160, 256, 32, 5
    fc, _, _ = make_cache(n_slots, 2, H, R, dtype, cuda, seed=41)
    x = torch.randn(B * S, H, generator=torch.Generator().manual_seed(15)).to(dtype).to(cuda)
    y = torch.randn(B * S, 2 * H, generator=torch.Generator().manual_seed(16)).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=17)
    tc = run_apply(x, y, fc, segs, [0, 1], [0, H])
    nat.set_option(nat.LF_OPT_REQUIRE_TC, 0)
    nat.set_option(nat.LF_OPT_FORCE_SIMT, 1)
    simt = run_apply(x, y, fc, segs, [0, 1], [0, H])
    d = (tc.float() - y.float())
    e = (simt.float() - y.float())
    rel = (d - e).norm() / e.norm()
    assert rel.item() < 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,R", [(32, 4), (48, 8), (256, 16), (100, 3)])
def test_simt_any_shape(cuda, dtype, H, R):
    """f32 (exact arithmetic) and shapes the tensor-core path does not tile."""
    B, S, n_slots = 3, 16, 4
    fc, a_of, b_of = make_cache(n_slots, 1, H, R, dtype, cuda, seed=H + R)
    x = torch.randn(B * S, H, generator=torch.Generator().manual_seed(18)).to(dtype).to(cuda)
    y = torch.randn(B * S, H, generator=torch.Generator().manual_seed(19)).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=20, lengths=[16, 5, 0])
    ours = run_apply(x, y, fc, segs, [0], [0]).cpu()
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs)
    check(ours, ref, y.cpu(), dtype)


def test_bad_slot_sets_status_without_fault(cuda):
    dtype = torch.bfloat16
    T, H, R = 256, 256, 16
    fc, _, _ = make_cache(2, 1, H, R, dtype, cuda)
    x = torch.randn(T, H, device=cuda, dtype=dtype)
    y = torch.randn(T, H, device=cuda, dtype=dtype)
    st = SegmentTable([0, 128], [128, 128], [1, 5], T, cuda)  # slot 5 is out of range
    ws = torch.empty(workspace_bytes(dtype, T, R, 1), dtype=torch.uint8, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = y.clone()
    lora_apply(x, out, fc, st, [0], [0], ws, status)
    torch.cuda.synchronize()
    assert status.item() & 1
    assert torch.equal(out[128:], y[128:])  # the bad segment got no delta


def test_large_cfg2_shape_vs_gathered_bmm(cuda):
    """(64, 256, 1024) bf16, r=16, 1,000 slots: the kernels against the reference's
    own GPU arithmetic (gather + bmm + add), on the same device."""
    dtype = torch.bfloat16
    B, S, H, R, n_slots = 64, 256, 1024, 16, 1000
    fc, _, _ = make_cache(n_slots, 1, H, R, dtype, cuda, seed=51, std=0.02)
    x = torch.randn(B * S, H, device=cuda, dtype=dtype)
    y = torch.randn(B * S, H, device=cuda, dtype=dtype)
    segs = segments_padded(B, S, n_slots, seed=52)
    ours = run_apply(x, y, fc, segs, [0], [0])
    slots = torch.tensor([k for _, _, k in segs], device=cuda)
    buf = fc.a
    a = buf[slots, 0, 0].view(B, H, R)
    b = buf[slots, 0, 1].view(B, R, H)
    out_a = torch.bmm(x.view(B, S, H), a)
    out_b = torch.bmm(out_a, b)
    ref = (y.view(B, S, H) + out_b).view(B * S, H)
    d1 = ours.float() - y.float()
    d2 = ref.float() - y.float()
    rel = (d1 - d2).norm() / d2.norm()
    assert rel.item() < 2e-2, rel.item()


@pytest.mark.parametrize("S", [100, 512])
def test_tc_tile_records_equal_segment_search(cuda, S):
    """Per-tile records (one read per CTA) and the binary search over the segment
    table (no records) give bit-identical results.  The shrink runs without a
    K split so both paths accumulate in the same order."""
    dtype = torch.bfloat16
    B, H, R, n_slots = 4, 256, 16, 6
    fc, _, _ = make_cache(n_slots, 3, H, R, dtype, cuda, seed=61)
    g = torch.Generator().manual_seed(S)
    lengths = torch.randint(1, S + 1, (B,), generator=g).tolist()
    x = torch.randn(B * S, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(B * S, 3 * H, generator=g).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=S, lengths=lengths)
    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 1)
    a = run_apply(x, y, fc, segs, [0, 1, 2], [0, H, 2 * H], records=True)
    b = run_apply(x, y, fc, segs, [0, 1, 2], [0, H, 2 * H], records=False)
    assert torch.equal(a, b)


def test_record_that_disagrees_with_segments_is_flagged(cuda):
    dtype = torch.bfloat16
    T, H, R = 256, 256, 16
    fc, _, _ = make_cache(4, 1, H, R, dtype, cuda)
    x = torch.randn(T, H, device=cuda, dtype=dtype)
    y = torch.randn(T, H, device=cuda, dtype=dtype)
    st = SegmentTable([0, 128], [128, 128], [1, 2], T, cuda)
    st.table[7] = 3  # tile 1's record names slot 3, the segment table says slot 2
    ws = torch.empty(workspace_bytes(dtype, T, R, 1), dtype=torch.uint8, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = y.clone()
    lora_apply(x, out, fc, st, [0], [0], ws, status)
    torch.cuda.synchronize()
    assert status.item() & 2
    assert torch.equal(out[128:], y[128:])       # that tile got no delta
    assert not torch.equal(out[:128], y[:128])   # the consistent tile did


def run_per_tile(fn, *args, **kw):
    """Run with the persistent kernels off and the shrink on one CTA per tile,
    so that every fp32 accumulation runs in the persistent kernels' order."""
    nat.set_option(nat.LF_OPT_PERSISTENT, 0)
    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 1)
    try:
        return fn(*args, **kw)
    finally:
        nat.set_option(nat.LF_OPT_PERSISTENT, 1)
        nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 0)


@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_tc_persistent_equals_per_tile_kernel(cuda, R):
    """The persistent shrink + expand (single-segment tiles) and the
    one-tile-per-CTA kernels run the same MMAs on the same operands in the same
    order: results are bit-identical."""
    dtype = torch.bfloat16
    B, S, H, n_slots = 6, 256, 512, 9
    fc, a_of, b_of = make_cache(n_slots, 3, H, R, dtype, cuda, seed=70 + R)
    g = torch.Generator().manual_seed(R)
    lengths = torch.randint(1, S + 1, (B,), generator=g).tolist()
    x = torch.randn(B * S, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(B * S, 3 * H, generator=g).to(dtype).to(cuda)
    segs = segments_padded(B, S, n_slots, seed=R, lengths=lengths)
    persistent = run_apply(x, y, fc, segs, [0, 1, 2], [0, H, 2 * H])
    per_tile = run_per_tile(run_apply, x, y, fc, segs, [0, 1, 2], [0, H, 2 * H])
    assert torch.equal(persistent, per_tile)
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs, col_offsets=[0, H, 2 * H], modules=[0, 1, 2])
    check(persistent.cpu(), ref, y.cpu(), dtype)


@pytest.mark.parametrize("R", [8, 16, 64])
def test_tc_persistent_shrink_with_multi_segment_tiles(cuda, R):
    """Packed segments: tiles holding one segment go to the persistent shrink,
    tiles holding several to the per-tile kernel, in one call; u equals the
    per-tile kernel's everywhere and is zero on rows outside every segment."""
    dtype = torch.bfloat16
    H, n_slots, n_mod = 512, 7, 2
    g = torch.Generator().manual_seed(300 + R)
    lengths = [300, 40, 17, 128, 256, 5, 90, 200]
    starts, t = [], 0
    for i, n in enumerate(lengths):
        starts.append(t)
        t += n + (3 if i % 3 == 0 else 0)  # a few uncovered rows between segments
    T = t + 50
    slots = torch.randint(0, n_slots, (len(lengths),), generator=g).tolist()
    fc, a_of, _ = make_cache(n_slots, n_mod, H, R, dtype, cuda, seed=90 + R)
    x = torch.randn(T, H, generator=g).to(dtype).to(cuda)
    st = SegmentTable(starts, lengths, slots, T, cuda)
    assert 0 < st.n_multi < st.n_tiles
    status = torch.zeros(1, dtype=torch.int32, device=cuda)

    def shrink():
        u = torch.full((n_mod, T, R), float("nan"), dtype=dtype, device=cuda)
        lora_shrink(x, u, fc, st, [0, 1], status)
        torch.cuda.synchronize()
        assert status.item() == 0, nat.decode_status(status.item())
        return u

    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 1)  # multi-segment tiles without a K split in both runs
    persistent = shrink()
    per_tile = run_per_tile(shrink)
    covered = torch.zeros(T, dtype=torch.bool, device=cuda)
    for s0, n in zip(starts, lengths):
        covered[s0 : s0 + n] = True
    tiles_touched = torch.zeros(T, dtype=torch.bool, device=cuda)
    for s0, n in zip(starts, lengths):
        tiles_touched[s0 // 128 * 128 : min(T, (s0 + n + 127) // 128 * 128)] = True
    # rows of a tile that holds a segment are written (0 where uncovered); others are never read
    assert torch.equal(persistent[:, tiles_touched], per_tile[:, tiles_touched])
    assert not persistent[:, covered].isnan().any()
    assert (persistent[:, tiles_touched & ~covered] == 0).all()
    xc = x.cpu().float()
    for m in range(n_mod):
        for s0, n, k in zip(starts, lengths, slots):
            ref = (xc[s0 : s0 + n] @ a_of(k, m).float()).to(dtype).float()
            got = persistent[m, s0 : s0 + n].cpu().float()
            assert (got - ref).abs().max().item() <= 2e-2 * max(ref.abs().max().item(), 1e-6)


@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_tc_persistent_packed_segments_equal_per_tile(cuda, R):
    """Packed rows (no padding, segments starting anywhere, several per tile):
    the persistent expand runs one sub-item per segment of a tile; the whole
    delta equals the one-tile-per-CTA kernels' bit for bit and the oracle's
    within tolerance."""
    dtype = torch.bfloat16
    H, n_slots = 512, 11
    g = torch.Generator().manual_seed(500 + R)
    lengths = torch.randint(1, 300, (24,), generator=g).tolist()
    lengths[3] = 1
    lengths[4] = 2
    slots = torch.randint(0, n_slots, (24,), generator=g).tolist()
    starts = [sum(lengths[:i]) for i in range(len(lengths))]
    T = sum(lengths)
    segs = list(zip(starts, lengths, slots))
    fc, a_of, b_of = make_cache(n_slots, 3, H, R, dtype, cuda, seed=600 + R)
    x = torch.randn(T, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(T, 3 * H, generator=g).to(dtype).to(cuda)
    st = SegmentTable(starts, lengths, slots, T, cuda)
    assert st.n_multi > 0
    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 1)
    persistent = run_apply(x, y, fc, segs, [0, 1, 2], [0, H, 2 * H])
    per_tile = run_per_tile(run_apply, x, y, fc, segs, [0, 1, 2], [0, H, 2 * H])
    assert torch.equal(persistent, per_tile)
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs, col_offsets=[0, H, 2 * H], modules=[0, 1, 2])
    check(persistent.cpu(), ref, y.cpu(), dtype)


@pytest.mark.parametrize("n_mod,R", [(1, 16), (3, 16), (3, 64), (2, 8)])
def test_tc_persistent_many_short_segments_per_tile(cuda, n_mod, R):
    """Tiles holding up to ~20 short segments with gaps between them: the
    persistent shrink multiplies each x K-block by several segments' A at once
    and needs several passes per tile; u (0 in the gaps) and the whole delta
    equal the one-tile-per-CTA kernels' bit for bit."""
    dtype = torch.bfloat16
    H, n_slots = 256, 13
    g = torch.Generator().manual_seed(700 + 10 * n_mod + R)
    lengths = torch.randint(1, 20, (60,), generator=g).tolist()
    gaps = torch.randint(0, 4, (60,), generator=g).tolist()
    starts, t = [], 0
    for n, gap in zip(lengths, gaps):
        t += gap
        starts.append(t)
        t += n
    T = t + 5
    slots = torch.randint(0, n_slots, (60,), generator=g).tolist()
    segs = list(zip(starts, lengths, slots))
    fc, a_of, b_of = make_cache(n_slots, n_mod, H, R, dtype, cuda, seed=800 + R)
    x = torch.randn(T, H, generator=g).to(dtype).to(cuda)
    y = torch.randn(T, n_mod * H, generator=g).to(dtype).to(cuda)
    mods, offs = list(range(n_mod)), [m * H for m in range(n_mod)]
    st = SegmentTable(starts, lengths, slots, T, cuda)
    assert st.n_multi > 0
    status = torch.zeros(1, dtype=torch.int32, device=cuda)

    def shrink():
        u = torch.full((n_mod, T, R), float("nan"), dtype=dtype, device=cuda)
        lora_shrink(x, u, fc, st, mods, status)
        torch.cuda.synchronize()
        assert status.item() == 0, nat.decode_status(status.item())
        return u

    nat.set_option(nat.LF_OPT_SHRINK_CLUSTER, 1)
    u_p = shrink()
    u_t = run_per_tile(shrink)
    covered = torch.zeros(T, dtype=torch.bool, device=cuda)
    for s0, n in zip(starts, lengths):
        covered[s0:s0 + n] = True
    touched = torch.zeros(T, dtype=torch.bool, device=cuda)
    for s0, n in zip(starts, lengths):
        touched[s0 // 128 * 128: min(T, (s0 + n + 127) // 128 * 128)] = True
    assert torch.equal(u_p[:, touched], u_t[:, touched])
    assert (u_p[:, touched & ~covered] == 0).all()
    persistent = run_apply(x, y, fc, segs, mods, offs)
    per_tile = run_per_tile(run_apply, x, y, fc, segs, mods, offs)
    assert torch.equal(persistent, per_tile)
    ref = segmented_apply(x.cpu(), y.cpu(), a_of, b_of, segs, col_offsets=offs, modules=mods)
    check(persistent.cpu(), ref, y.cpu(), dtype)


def test_tc_persistent_expand_many_items_per_cta(cuda):
    """bge-m3 q/k/v shape: 256 tiles x 3 modules x 8 column blocks = 6,144 work
    items over at most 148 CTAs, so every CTA cycles its stage ring many times;
    the persistent shrink likewise streams 16 K blocks for each of 256 tiles."""
    dtype = torch.bfloat16
    B, S, H, R, n_slots = 64, 512, 1024, 16, 300
    fc, a_of, b_of = make_cache(n_slots, 3, H, R, dtype, cuda, seed=81, std=0.02)
    x = torch.randn(B * S, H, device=cuda, dtype=dtype)
    y = torch.randn(B * S, 3 * H, device=cuda, dtype=dtype)
    lengths = torch.randint(32, S + 1, (B,), generator=torch.Generator().manual_seed(3)).tolist()
    segs = segments_padded(B, S, n_slots, seed=82, lengths=lengths)
    st = SegmentTable([s for s, _, _ in segs], [l for _, l, _ in segs], [k for _, _, k in segs], B * S, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    u = torch.empty(3, B * S, R, dtype=dtype, device=cuda)
    lora_shrink(x, u, fc, st, [0, 1, 2], status)
    # expand: persistent vs per-tile on the same u
    persistent = y.clone()
    lora_expand(u, persistent, fc, st, [0, 1, 2], [0, H, 2 * H], True, status)
    per_tile = y.clone()
    run_per_tile(lora_expand, u, per_tile, fc, st, [0, 1, 2], [0, H, 2 * H], True, status)
    torch.cuda.synchronize()
    assert status.item() == 0, nat.decode_status(status.item())
    assert torch.equal(persistent, per_tile)
    # the whole delta against the oracle on a few sequences
    pick = [0, 17, 63]
    sub = [segs[i] for i in pick]
    rows = torch.cat([torch.arange(s, s + l) for s, l, _ in sub])
    local, t0 = [], 0
    for s, l, k in sub:
        local.append((t0, l, k))
        t0 += l
    ref = segmented_apply(x.cpu()[rows], y.cpu()[rows], a_of, b_of, local, col_offsets=[0, H, 2 * H],
                          modules=[0, 1, 2])
    check(persistent.cpu()[rows], ref, y.cpu()[rows], dtype)


@pytest.mark.parametrize("R", [8, 16, 32, 64])
def test_shrink_one_copy_for_evenly_spaced_modules(cuda, R):
    """Modules whose cache indices step evenly ([0, 1, 2], [1, 3]) have their A boxes
    staged by one 4-D copy per segment; any other order takes one copy per module.
    Both give the same bits for every module."""
    dtype, H, n_slots = torch.bfloat16, 512, 7
    fc, _, _ = make_cache(n_slots, 4, H, R, dtype, cuda, seed=R)
    g = torch.Generator().manual_seed(R)
    lens = torch.randint(1, 300, (12,), generator=g).tolist()
    slots = torch.randint(0, n_slots, (12,), generator=g).tolist()
    starts = [sum(lens[:i]) for i in range(12)]
    T = sum(lens)
    st = SegmentTable(starts, lens, slots, T, cuda)
    x = torch.randn(T, H, device=cuda, dtype=dtype)
    for mods, other in (([0, 1, 2], [2, 0, 1]), ([1, 3], [3, 1])):
        u1 = torch.empty(len(mods), T, R, dtype=dtype, device=cuda)
        u2 = torch.empty(len(mods), T, R, dtype=dtype, device=cuda)
        lora_shrink(x, u1, fc, st, mods)
        lora_shrink(x, u2, fc, st, other)
        torch.cuda.synchronize()
        for i, m in enumerate(mods):
            assert torch.equal(u1[i], u2[other.index(m)]), (mods, m)
