"""``lf_linear_lora``: the projection GEMM with the per-row LoRA delta in its
accumulator, against the reference's order of operations on the existing entry
points (``F.linear`` with its bias, then ``lf_lora_apply`` adding the rounded
delta in place) and against an f32 computation.

The fused kernel rounds ``x W^T + b + delta`` once; the reference rounds the
projection and the delta apart and then their sum, so the two agree within the
bf16/f16 serving tolerance (2e-2 relative, max error over max magnitude), and
the fused result is at least as close to the f32 value as the reference's.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from latefuse_b200 import _native as nat
from latefuse_b200.encoder_ops import ACT_GELU
from latefuse_b200.lora import (FactorCache, SegmentTable, blocked_u, linear_lora, lora_apply, lora_shrink,
                                lora_shrink_blocked, workspace_bytes)

pytestmark = pytest.mark.gpu


def make_cache(n_slots, n_mod, H, R, dtype, dev, seed=0, std=0.05):
    g = torch.Generator(device="cpu").manual_seed(seed)
    buf = (torch.randn(n_slots, n_mod, 2, H * R, generator=g) * std).to(dtype).to(dev)
    return FactorCache(a=buf, b=buf, a_offset=0, b_offset=H * R, a_slot_stride=buf.stride(0),
                       b_slot_stride=buf.stride(0), a_module_stride=buf.stride(1), b_module_stride=buf.stride(1),
                       n_slots=n_slots, hidden=H, rank=R), buf


def packed_segments(n_rows, n_slots, seed, max_len=400, gap_every=0):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (n_rows,), generator=g).tolist()
    slots = sorted(torch.randint(0, n_slots, (n_rows,), generator=g).tolist())
    starts, lengths, sl = [], [], []
    pos = 0
    for i, (n, s) in enumerate(zip(lens, slots)):
        if gap_every and i % gap_every == 1:
            pos += 37  # tokens in no segment
        if sl and sl[-1] == s and not gap_every:
            lengths[-1] += n
        else:
            starts.append(pos)
            lengths.append(n)
            sl.append(s)
        pos += n
    return starts, lengths, sl, pos + (5 if gap_every else 0)


def check(fused, ref, exact):
    f, r, e = fused.float(), ref.float(), exact.float()
    assert (f - r).abs().max().item() <= 2e-2 * r.abs().max().item()
    assert ((f - r).norm() / r.norm()).item() < 4e-3
    assert (f - e).norm().item() <= (r - e).norm().item() * 1.05


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("R", [16, 32, 64])
@pytest.mark.parametrize("n_mod", [3, 1])
def test_linear_lora_matches_reference_order(cuda, dtype, R, n_mod):
    H, n_slots = 1024 if n_mod == 1 else 512, 37
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(30, n_slots, seed=R + n_mod)
    fc, buf = make_cache(n_slots, n_mod + 1, H, R, dtype, dev, seed=R)
    st = SegmentTable(starts, lengths, slots, T, dev)
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(T, H, generator=g).to(dtype).to(dev)
    N = n_mod * H
    W = (torch.randn(N, H, generator=g) * H ** -0.5).to(dtype).to(dev)
    b = torch.randn(N, generator=g).to(dtype).to(dev)
    modules = list(range(1, n_mod + 1))  # not the cache's first module
    offs = [i * H for i in range(n_mod)]
    u = blocked_u(n_mod, T, st.n_segs, R, dtype, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    lora_shrink_blocked(x, u, fc, st, modules, status)
    fused = linear_lora(x, W, b, u, fc, st, modules, H, status=status)
    ref = F.linear(x, W, b)
    ws = torch.empty(workspace_bytes(dtype, T, R, n_mod), dtype=torch.uint8, device=dev)
    lora_apply(x, ref, fc, st, modules, offs, ws, status)
    torch.cuda.synchronize()
    assert status.item() == 0, nat.decode_status(status.item())
    # f32: the projection plus each row's delta from its own slot's factors
    exact = F.linear(x.float(), W.float(), b.float())
    slot_of = torch.empty(T, dtype=torch.long)
    for s0, n, k in zip(starts, lengths, slots):
        slot_of[s0:s0 + n] = k
    for i, m in enumerate(modules):
        A = buf[:, m, 0].view(n_slots, H, R).float()[slot_of.to(dev)]
        B = buf[:, m, 1].view(n_slots, R, H).float()[slot_of.to(dev)]
        exact[:, i * H:(i + 1) * H] += torch.bmm(torch.bmm(x.float()[:, None], A), B)[:, 0]
    check(fused, ref, exact)


def test_linear_lora_rows_outside_segments_and_partial_tiles(cuda):
    """Tokens between segments get the plain projection; segments start and end
    inside tiles, several per tile; the last tile is partial."""
    dtype, H, R, n_slots = torch.bfloat16, 1024, 16, 9
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(40, n_slots, seed=3, max_len=90, gap_every=3)
    fc, _ = make_cache(n_slots, 1, H, R, dtype, dev, seed=1)
    st = SegmentTable(starts, lengths, slots, T, dev)
    x = torch.randn(T, H, device=dev, dtype=dtype)
    W = (torch.randn(H, H, device=dev) * H ** -0.5).to(dtype)
    u = blocked_u(1, T, st.n_segs, R, dtype, dev)
    lora_shrink_blocked(x, u, fc, st, [0])
    fused = linear_lora(x, W, None, u, fc, st, [0], H)
    ref = F.linear(x, W)
    ws = torch.empty(workspace_bytes(dtype, T, R, 1), dtype=torch.uint8, device=dev)
    lora_apply(x, ref, fc, st, [0], [0], ws)
    torch.cuda.synchronize()
    assert (fused.float() - ref.float()).abs().max().item() <= 2e-2 * ref.float().abs().max().item()
    covered = torch.zeros(T, dtype=torch.bool)
    for s0, n in zip(starts, lengths):
        covered[s0:s0 + n] = True
    plain = F.linear(x, W)
    gap = (~covered).to(dev)
    assert gap.any()
    torch.testing.assert_close(fused[gap].float(), plain[gap].float(), atol=2e-2, rtol=2e-2)


def test_linear_lora_rejections(cuda):
    dev = torch.device("cuda")
    fc, _ = make_cache(2, 1, 512, 8, torch.bfloat16, dev)
    st = SegmentTable([0], [100], [0], 100, dev)
    x = torch.randn(100, 512, device=dev, dtype=torch.bfloat16)
    W = torch.randn(512, 512, device=dev, dtype=torch.bfloat16)
    u = blocked_u(1, 100, 1, 8, torch.bfloat16, dev)
    with pytest.raises(nat.NativeLibraryError, match="rank 8"):
        linear_lora(x, W, None, u, fc, st, [0], 512)


@pytest.mark.parametrize("R", [16, 32, 64])
def test_blocked_shrink_is_the_dense_shrink_reordered(cuda, R):
    """Block (tile, segment) holds the dense shrink's rows of that segment, bit for
    bit, and zeros in the tile's other rows (including rows past the last token)."""
    dtype, H, n_slots = torch.bfloat16, 512, 11
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(20, n_slots, seed=R)
    fc, _ = make_cache(n_slots, 2, H, R, dtype, dev, seed=R)
    st = SegmentTable(starts, lengths, slots, T, dev)
    x = torch.randn(T, H, device=dev, dtype=dtype)
    dense = torch.empty(2, T, R, dtype=dtype, device=dev)
    lora_shrink(x, dense, fc, st, [0, 1])
    ub = blocked_u(2, T, st.n_segs, R, dtype, dev)
    lora_shrink_blocked(x, ub, fc, st, [0, 1])
    torch.cuda.synchronize()
    n_rt = (T + 127) // 128
    n_blk = n_rt + st.n_segs
    # element (m, blk, g, q, r8, e) -> tile row 8 g + r8, column 8 q + e
    blocks = ub.view(2, n_blk, 16, R // 8, 8, 8).permute(0, 1, 2, 4, 3, 5).reshape(2, n_blk, 128, R).cpu()
    d = dense.cpu()
    checked = 0
    for g, (s0, n) in enumerate(zip(starts, lengths)):
        for tb in range(s0 // 128, (s0 + n - 1) // 128 + 1):
            blk = blocks[:, tb + g]
            rows = torch.arange(tb * 128, tb * 128 + 128)
            inside = (rows >= s0) & (rows < s0 + n)
            assert torch.equal(blk[:, inside], d[:, rows[inside]])
            assert not blk[:, ~inside].any()
            checked += 1
    assert checked >= n_rt


def test_shrink_skips_malformed_tile_records(cuda):
    """A tile record past the tokens or naming a segment outside the table sets
    LF_STATUS_BAD_SEGMENT and writes nothing: u stays inside its buffer (dense and
    blocked layouts), and the well-formed records are still computed."""
    dtype, H, R, n_slots = torch.bfloat16, 512, 16, 5
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(8, n_slots, seed=9, max_len=200)
    fc, _ = make_cache(n_slots, 2, H, R, dtype, dev, seed=9)
    st = SegmentTable(starts, lengths, slots, T, dev)
    x = torch.randn(T, H, device=dev, dtype=dtype)
    good_dense = torch.empty(2, T, R, dtype=dtype, device=dev)
    lora_shrink(x, good_dense, fc, st, [0, 1])
    assert st.n_tiles >= 3
    st.table[0] = 1 << 20        # record 0: a tile far past the last token
    st.table[4 + 1] = -5         # record 1: first segment outside the table
    n_u = 2 * T * R
    canary = torch.full((n_u + 4096,), 3.0, dtype=dtype, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    lora_shrink(x, canary[:n_u].view(2, T, R), fc, st, [0, 1], status=status)
    n_b = blocked_u(2, T, st.n_segs, R, dtype, dev).numel()
    canary_b = torch.full((n_b + 4096,), 3.0, dtype=dtype, device=dev)
    status_b = torch.zeros(1, dtype=torch.int32, device=dev)
    lora_shrink_blocked(x, canary_b[:n_b], fc, st, [0, 1], status=status_b)
    torch.cuda.synchronize()
    assert status.item() & nat.LF_STATUS_BAD_SEGMENT and status_b.item() & nat.LF_STATUS_BAD_SEGMENT
    assert (canary[n_u:] == 3.0).all() and (canary_b[n_b:] == 3.0).all()
    # rows of the well-formed records (tiles 2 and later) are unchanged
    rec = st.host[: 4 * st.n_tiles].view(-1, 4)
    row2 = int(rec[2, 0]) * 128
    dense = canary[:n_u].view(2, T, R)
    assert torch.equal(dense[:, row2:], good_dense[:, row2:])


@pytest.mark.parametrize("corrupt", ["slot", "segment", "range"])
def test_fused_gemm_reports_malformed_pair_table(cuda, corrupt):
    """A pair naming a slot outside the cache (LF_STATUS_BAD_SLOT), a segment outside
    the table, or a tile whose pair range is not ascending (LF_STATUS_BAD_SEGMENT)
    is reported and the launch ends normally; the other tiles keep their delta."""
    dtype, H, R, n_slots = torch.bfloat16, 512, 16, 4
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(6, n_slots, seed=21, max_len=300)
    fc, _ = make_cache(n_slots, 1, H, R, dtype, dev, seed=21)
    st = SegmentTable(starts, lengths, slots, T, dev)
    x = torch.randn(T, H, device=dev, dtype=dtype)
    W = torch.randn(H, H, device=dev, dtype=dtype) * H ** -0.5
    u = blocked_u(1, T, st.n_segs, R, dtype, dev)
    lora_shrink_blocked(x, u, fc, st, [0])
    good = linear_lora(x, W, None, u, fc, st, [0], H)
    n_q = (T + 255) // 256  # 256-token tiles, one per CTA pair
    assert n_q >= 2
    tp = 4 * st.n_tiles + 3 * st.n_segs
    pairs = tp + n_q + 1
    last = n_q - 1  # a tile whose entries are changed; tile 0 is left alone
    q_last = int(st.host[tp + last])
    if corrupt == "slot":
        st.table[pairs + 3 * q_last + 1] = n_slots + 7
        want = nat.LF_STATUS_BAD_SLOT
    elif corrupt == "segment":
        st.table[pairs + 3 * q_last] = -3
        want = nat.LF_STATUS_BAD_SEGMENT
    else:
        st.table[tp + last] = 1 << 30
        want = nat.LF_STATUS_BAD_SEGMENT
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = linear_lora(x, W, None, u, fc, st, [0], H, status=status)
    torch.cuda.synchronize()
    assert status.item() & want
    assert torch.equal(out[:256], good[:256])


def _u_rows(u, st, n_mod, R):
    """The blocked u as {(module, tile, segment): 128 x R block}, for the blocks the pair
    table names (the others are never read)."""
    n_blk = (st.n_tokens + 127) // 128 + st.n_segs
    blocks = u.view(n_mod, n_blk, 128 * R)
    tp = 4 * st.n_tiles + 3 * st.n_segs
    n_q = (st.n_tokens + 255) // 256
    h = st.host.tolist()
    out = {}
    for q in range(n_q):
        for e in range(h[tp + q], h[tp + q + 1]):
            j, _, mask = h[tp + n_q + 1 + 3 * e: tp + n_q + 4 + 3 * e]
            for r in range(2):
                if (mask >> r) & 1:
                    for m in range(n_mod):
                        out[(m, 2 * q + r, j)] = blocks[m, 2 * q + r + j]
    return out


@pytest.mark.parametrize("R,n_mod,max_len", [(16, 3, 400), (16, 3, 40), (32, 3, 300), (64, 1, 300), (16, 1, 25),
                                             (16, 3, 2000), (16, 1, 3000)])
def test_shrink_in_the_gemm_launch_matches_the_two_launches(cuda, R, n_mod, max_len):
    """``lf_linear_lora_shrink`` computes u in the GEMM's own launch: its u blocks and its
    output against ``lf_lora_shrink_blocked`` + ``lf_linear_lora`` on the same inputs.
    Short segments put many segments in one 256-token block (several shrink passes);
    the small batches give several CTA pairs each part of one row block (each computes
    that block's u), the long ones give pairs ranges that cross row blocks."""
    dtype, H, n_slots = torch.bfloat16, 1024 if n_mod == 1 else 512, 37
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(30 if max_len > 100 else 80, n_slots, seed=R + max_len,
                                                max_len=max_len)
    fc, _ = make_cache(n_slots, n_mod + 1, H, R, dtype, dev, seed=R)
    st = SegmentTable(starts, lengths, slots, T, dev)
    g = torch.Generator(device="cpu").manual_seed(9)
    x = torch.randn(T, H, generator=g).to(dtype).to(dev)
    N = n_mod * H
    W = (torch.randn(N, H, generator=g) * H ** -0.5).to(dtype).to(dev)
    b = torch.randn(N, generator=g).to(dtype).to(dev)
    modules = list(range(1, n_mod + 1))
    u_two = blocked_u(n_mod, T, st.n_segs, R, dtype, dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    lora_shrink_blocked(x, u_two, fc, st, modules, status)
    two = linear_lora(x, W, b, u_two, fc, st, modules, H, status=status)
    u_one = torch.full_like(u_two, float("nan"))  # every block the table names must be written
    one = linear_lora(x, W, b, u_one, fc, st, modules, H, status=status, shrink=True)
    # the transposed weight (read in the delta factors' operand form), with and without
    # the shrink in the launch
    Wt = W.t().contiguous()
    two_kn = linear_lora(x, None, b, u_two, fc, st, modules, H, status=status, weight_t=Wt)
    one_kn = linear_lora(x, None, b, torch.full_like(u_two, float("nan")), fc, st, modules, H, status=status,
                         shrink=True, weight_t=Wt)
    torch.cuda.synchronize()
    assert status.item() == 0, nat.decode_status(status.item())
    check(two_kn, two, two)
    check(one_kn, two, two)
    got, want = _u_rows(u_one, st, n_mod, R), _u_rows(u_two, st, n_mod, R)
    assert got.keys() == want.keys()
    for k in want:
        assert not torch.isnan(got[k]).any(), k
        assert (got[k].float() - want[k].float()).abs().max().item() <= 2e-2 * want[k].float().abs().max().item() + 1e-6
    check(one, two, two)


@pytest.mark.parametrize("shrink", [False, True])
def test_lora_gemm_with_gelu_is_the_gelu_of_the_lora_gemm(cuda, shrink):
    """act = GELU on the LoRA GEMM: the epilogue's GELU applied to the same rounded sum the
    plain LoRA GEMM returns (within one bf16 ulp; the formula's f32 cancellation for
    inputs below about -4 allowed for as in the plain GEMM's test)."""
    dtype, H, R, n_slots = torch.bfloat16, 512, 16, 37
    dev = torch.device("cuda")
    starts, lengths, slots, T = packed_segments(30, n_slots, seed=5)
    fc, _ = make_cache(n_slots, 4, H, R, dtype, dev, seed=5)
    st = SegmentTable(starts, lengths, slots, T, dev)
    g = torch.Generator(device="cpu").manual_seed(6)
    x = torch.randn(T, H, generator=g).to(dtype).to(dev)
    W = (torch.randn(3 * H, H, generator=g) * H ** -0.5).to(dtype).to(dev)
    b = torch.randn(3 * H, generator=g).to(dtype).to(dev)
    mods = [1, 2, 3]
    u = blocked_u(3, T, st.n_segs, R, dtype, dev)
    if not shrink:
        lora_shrink_blocked(x, u, fc, st, mods)
    plain = linear_lora(x, W, b, u, fc, st, mods, H, shrink=shrink).float()
    act = linear_lora(x, W, b, u, fc, st, mods, H, act=ACT_GELU, shrink=shrink)
    want = (plain * 0.5 * (1.0 + torch.erf(plain * 0.70710678118654752440))).to(dtype)
    lo, hi = act.view(torch.int16).int(), want.view(torch.int16).int()
    dist = (torch.where(lo < 0, -(lo & 0x7FFF), lo) - torch.where(hi < 0, -(hi & 0x7FFF), hi)).abs()
    near = (act.float() - want.float()).abs() <= plain.abs() * 2.0 ** -22
    assert not ((dist > 1) & ~near).any()
    assert (dist != 0).float().mean().item() < 2e-3


def test_shrink_in_the_gemm_launch_rejects_what_it_cannot_stage(cuda):
    dtype, H, R = torch.bfloat16, 512, 64
    dev = torch.device("cuda")
    fc, _ = make_cache(4, 3, H, R, dtype, dev)
    st = SegmentTable([0], [300], [1], 300, dev)
    x = torch.randn(300, H, device=dev, dtype=dtype)
    W = torch.randn(3 * H, H, device=dev, dtype=dtype)
    u = blocked_u(3, 300, 1, R, dtype, dev)
    with pytest.raises(nat.NativeLibraryError, match="above 128"):  # 3 modules x rank 64
        linear_lora(x, W, None, u, fc, st, [0, 1, 2], H, shrink=True)
