"""The late-fusion LoRA delta on the GPU, and the reference's ``LoraOps`` API over it.

For a mixed-tenant batch every token row ``t`` belongs to one adapter slot, and
each targeted projection output gets

    y[t] += B_slot(t) (A_slot(t) x[t])

The reference computes this with a per-layer ``torch.cat``/``index_select``
gather of the per-row factors followed by two ``torch.bmm`` calls and an add
(``src/latefuse/ops/lora.py:57,75``, ``src/latefuse/model/hf_wrapper.py:213-217``).
Here one :func:`lora_apply` call runs the sm_100a kernels, which read each
tenant's factors in place from the slot cache: for one module, a single kernel
that keeps the shrink output on chip and adds the delta to y in L2; for several
modules sharing x, a shrink launch and an expand launch (same bits either way).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from latefuse_b200 import _native as nat
from latefuse_b200.config import LoraServingConfig


# ---------------------------------------------------------------------------
# segment tables
# ---------------------------------------------------------------------------
class SegmentTable:
    """Runs of consecutive tokens that share one adapter slot, as device int32 arrays.

    For a padded ``(B, S)`` batch row ``b`` is the segment ``{b*S, len_b, slot_b}``
    with ``len_b = S`` (every position gets its delta, as in the reference) or the
    row's real length when padding is skipped (right-padded rows only: real
    tokens first).  Skipping padding changes no real token's output, because
    padded keys are masked out of attention and every other op is per token.

    The table also carries one record per 128-token row tile that holds any
    segment token -- ``{tile, first overlapping segment, number of overlapping
    segments, slot of the first}`` -- so the kernels launch nothing for tiles of
    pure padding and issue every load of a tile after one 16-byte read.
    Everything lives in one int32 buffer, ``[records | starts | lengths | slots]``,
    copied to the device once per batch.
    """

    def __init__(self, starts, lengths, slots, n_tokens: int, device: torch.device, records: bool = True):
        starts, lengths, slots = list(starts), list(lengths), list(slots)
        if not (len(starts) == len(lengths) == len(slots)):
            raise ValueError("starts, lengths and slots must have equal length")
        self.n_segs = len(starts)
        self.n_tokens = int(n_tokens)
        self.device = torch.device(device)
        self.use_records = records
        records = _tile_records(starts, lengths, slots) if records else []
        self.n_tiles = len(records) // 4
        self.n_multi = sum(1 for i in range(2, len(records), 4) if records[i] != 1)
        pairs = _pair_tiles(starts, lengths, slots, self.n_tokens) if self.use_records else []
        self.host = torch.tensor(records + starts + lengths + slots + pairs, dtype=torch.int32)
        if self.device.type == "cuda":
            self.table = self.host.pin_memory().to(self.device, non_blocking=True)
        else:
            self.table = self.host.clone()
        self.slots = slots
        self.real_tokens = int(sum(max(0, n) for n in lengths))

    @classmethod
    def for_padded(cls, slots, seq_len: int, device, lengths=None) -> SegmentTable:
        B = len(slots)
        lens = [seq_len] * B if lengths is None else [int(min(seq_len, max(0, n))) for n in lengths]
        return cls([b * seq_len for b in range(B)], lens, slots, B * seq_len, device)

    def ptrs(self) -> tuple[int, int, int, int, int, int]:
        """(seg_start, seg_len, seg_slot, tile records, n_tiles, n_multi) for the C ABI."""
        base = self.table.data_ptr()
        r = 16 * self.n_tiles
        n = self.n_segs
        if not self.use_records:
            return base, base + 4 * n, base + 8 * n, None, 0, 0
        return base + r, base + r + 4 * n, base + r + 8 * n, base, self.n_tiles, self.n_multi

    def pair_ptrs(self) -> tuple[int, int]:
        """(tile_pairs, pairs) for ``lf_linear_lora``: per 256-token tile q, the
        segments with tokens in it are entries ``tile_pairs[q] .. tile_pairs[q + 1]``
        of ``pairs`` (three int32 each: segment, slot, and a mask of the tile's
        128-token halves the segment has tokens in), in segment order.  Built with
        the tile records."""
        if not self.use_records:
            raise ValueError("the pair table is built with the tile records")
        off = self.table.data_ptr() + 16 * self.n_tiles + 12 * self.n_segs
        n_q = (self.n_tokens + 255) // 256
        return off, off + 4 * (n_q + 1)


def _pair_tiles(starts, lengths, slots, n_tokens: int) -> list[int]:
    """``[offsets (n_q + 1) | entries (3 per entry)]``: for every 256-token tile q (the
    rows one CTA pair of ``lf_linear_lora`` computes), the segments with tokens in
    it, in segment order, as ``{segment, slot, mask}`` with mask bit r set when the
    segment has tokens in the tile's 128-token half r (128-token tile 2q + r);
    segments of no tokens are left out."""
    tile = nat.TILE_TOKENS
    n_q = (int(n_tokens) + 2 * tile - 1) // (2 * tile)
    st = np.asarray(starts, dtype=np.int64)
    ln = np.asarray(lengths, dtype=np.int64)
    seg = np.nonzero(ln > 0)[0]
    if seg.size == 0:
        return [0] * (n_q + 1)
    # one (segment, 128-token tile) entry per tile a segment touches
    t0 = st[seg] // tile
    nt = (st[seg] + ln[seg] - 1) // tile - t0 + 1
    seg_of = np.repeat(seg, nt)
    tile_of = np.repeat(t0, nt) + np.arange(int(nt.sum())) - np.repeat(np.cumsum(nt) - nt, nt)
    q_of, bit = tile_of // 2, np.left_shift(1, tile_of % 2)
    # merge the two halves' entries of one (256-token tile, segment)
    key = q_of * (int(seg.max()) + 1) + seg_of
    order = np.argsort(key, kind="stable")
    key, q_of, seg_of, bit = key[order], q_of[order], seg_of[order], bit[order]
    uniq, first = np.unique(key, return_index=True)
    mask = np.bitwise_or.reduceat(bit, first)
    q_u, seg_u = q_of[first], seg_of[first]
    begin = np.searchsorted(q_u, np.arange(n_q + 1), side="left")
    entries = np.stack([seg_u, np.asarray(slots, dtype=np.int64)[seg_u], mask], axis=1)
    return begin.tolist() + entries.reshape(-1).tolist()


def _tile_records(starts, lengths, slots) -> list[int]:
    """Flattened ``{tile, first segment, segment count, first slot}`` records of the
    tiles that hold segment tokens (segments sorted by start, not overlapping):
    single-segment tiles first, in tile order, then the tiles with several segments."""
    tile = nat.TILE_TOKENS
    st = np.asarray(starts, dtype=np.int64)
    ln = np.asarray(lengths, dtype=np.int64)
    seg = np.nonzero(ln > 0)[0]
    if seg.size == 0:
        return []
    t0 = st[seg] // tile
    nt = (st[seg] + ln[seg] - 1) // tile - t0 + 1
    # one (segment, tile) entry per tile a segment touches, by segment then tile
    seg_of = np.repeat(seg, nt)
    tile_of = np.repeat(t0, nt) + np.arange(int(nt.sum())) - np.repeat(np.cumsum(nt) - nt, nt)
    order = np.argsort(tile_of, kind="stable")  # by tile; within a tile by segment
    tiles, first_idx, n_touch = np.unique(tile_of[order], return_index=True, return_counts=True)
    first = seg_of[order][first_idx]
    # the count spans segment indices first..last (an empty segment in between counts)
    count = seg_of[order][first_idx + n_touch - 1] - first + 1
    slot_arr = np.asarray(slots, dtype=np.int64)
    recs = np.stack([tiles, first, count, slot_arr[first]], axis=1)
    # tiles with one segment first (the cheapest work first), then the rest, each in tile order
    recs = recs[np.argsort(count != 1, kind="stable")]
    return recs.reshape(-1).tolist()


# ---------------------------------------------------------------------------
# cache views
# ---------------------------------------------------------------------------
@dataclass
class FactorCache:
    """Where the shrink (A, hidden x rank) and expand (B, rank x hidden) factors of
    every slot live, for one layer.  Strides are in elements.

    ``a``/``b`` are tensors whose ``data_ptr()`` is the address of slot 0, module 0.
    """

    a: Tensor
    b: Tensor
    a_offset: int          # element offset of (slot 0, module 0) from a.data_ptr()
    b_offset: int
    a_slot_stride: int
    b_slot_stride: int
    a_module_stride: int
    b_module_stride: int
    n_slots: int
    hidden: int
    rank: int

    @property
    def a_ptr(self) -> int:
        return self.a.data_ptr() + self.a_offset * self.a.element_size()

    @property
    def b_ptr(self) -> int:
        return self.b.data_ptr() + self.b_offset * self.b.element_size()


def _seg_args(segs: SegmentTable) -> tuple:
    s, l, k, t, nt, nm = segs.ptrs()
    return s, l, k, segs.n_segs, t, nt, nm


def workspace_bytes(dtype: torch.dtype, n_tokens: int, rank: int, n_modules: int) -> int:
    return int(nat.lib().lf_lora_workspace_bytes(nat.dtype_code(dtype), n_tokens, rank, n_modules))


def _rows(t: Tensor) -> tuple[Tensor, int]:
    """``t`` as a 2-D tensor of rows with unit column stride, and its row stride."""
    if t.dim() == 2 and t.stride(-1) == 1:
        return t, t.stride(0)
    t = t.contiguous()
    return t.reshape(-1, t.shape[-1]), t.shape[-1]


def lora_apply(x: Tensor, y: Tensor, cache: FactorCache, segs: SegmentTable, modules, y_col_offsets,
               workspace: Tensor, status: Tensor | None = None) -> None:
    """``y[:, off_m : off_m + H] += B(A x)`` for each op module, in place, on the current stream.

    Args:
        x:  ``(..., H)`` input of the projections (the rows of one batch).
        y:  ``(..., C)`` projection output(s), updated in place; module ``m`` owns
            columns ``y_col_offsets[m] : y_col_offsets[m] + H``.
        modules: cache module indices, one per op module (<= 4).
    """
    dev = nat.require_cuda(x, y, workspace, segs.table)
    x2, ldx = _rows(x)
    if not y.is_contiguous() and y.stride(-1) != 1:
        raise ValueError("y must have unit stride in its last dimension")
    y2 = y.reshape(-1, y.shape[-1])
    if y2.data_ptr() != y.data_ptr():
        raise ValueError("y must be viewable as rows without a copy")
    ldy = y2.stride(0)
    n = len(modules)
    rc = nat.lib().lf_lora_apply(
        nat.stream_ptr(dev), nat.dtype_code(x.dtype),
        x2.data_ptr(), ldx, y2.data_ptr(), ldy, x2.shape[0], cache.hidden, cache.rank,
        cache.a_ptr, cache.a_slot_stride, cache.a_module_stride,
        cache.b_ptr, cache.b_slot_stride, cache.b_module_stride,
        cache.n_slots, n, nat.i32_array(modules), nat.i64_array(y_col_offsets),
        *_seg_args(segs),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        nat.ptr(status))
    nat.check(rc, "lf_lora_apply")


def lora_apply_into(x: Tensor, y: Tensor, cache: FactorCache, segs: SegmentTable, modules, y_col_offsets,
                    workspace: Tensor, status: Tensor | None = None, residual: Tensor | None = None,
                    bias: Tensor | None = None) -> None:
    """``y[:, off_m : off_m + H] = round(round(residual + bias) + B(A x))`` for each op
    module (``residual``/``bias`` optional), written for every token, so that a
    ``y.addmm_(x, W.t())`` afterwards gives the biased projection plus delta (plus
    residual) with the projection output written once.  The segments must cover
    every token and carry tile records (a packed batch's table does); the op
    modules must cover every column of ``y`` the caller reads.
    """
    dev = nat.require_cuda(x, y, workspace, segs.table, residual, bias)
    if not segs.use_records or segs.real_tokens != x.reshape(-1, x.shape[-1]).shape[0]:
        raise ValueError("lora_apply_into needs tile records and segments covering every token")
    x2, ldx = _rows(x)
    y2 = y.reshape(-1, y.shape[-1])
    if y2.data_ptr() != y.data_ptr() or y2.stride(-1) != 1:
        raise ValueError("y must be viewable as rows without a copy")
    r2, ldr = (None, 0)
    if residual is not None:
        r2 = residual.reshape(-1, residual.shape[-1])
        if r2.stride(-1) != 1:
            raise ValueError("residual rows must be contiguous")
        ldr = r2.stride(0)
    b = None if bias is None else (bias if bias.dtype == y.dtype else bias.to(y.dtype)).contiguous()
    n = len(modules)
    rc = nat.lib().lf_lora_apply_into(
        nat.stream_ptr(dev), nat.dtype_code(x.dtype),
        x2.data_ptr(), ldx, nat.ptr(r2), ldr, nat.ptr(b), y2.data_ptr(), y2.stride(0), x2.shape[0],
        cache.hidden, cache.rank,
        cache.a_ptr, cache.a_slot_stride, cache.a_module_stride,
        cache.b_ptr, cache.b_slot_stride, cache.b_module_stride,
        cache.n_slots, n, nat.i32_array(modules), nat.i64_array(y_col_offsets),
        *_seg_args(segs),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        nat.ptr(status))
    nat.check(rc, "lf_lora_apply_into")


def blocked_u(n_modules: int, n_tokens: int, n_segs: int, rank: int, dtype: torch.dtype, device) -> Tensor:
    """An empty shrink output in the blocked layout of :func:`lora_shrink_blocked`:
    one 128 x rank block per (token tile, segment) pair, per module."""
    return torch.empty(n_modules, ((n_tokens + 127) // 128 + n_segs) * 128, rank, dtype=dtype, device=device)


def _blocked_elems(n_modules: int, n_tokens: int, n_segs: int, rank: int) -> int:
    return n_modules * ((n_tokens + 127) // 128 + n_segs) * 128 * rank


def fused_shrink_ok(modules, rank: int) -> bool:
    """Whether :func:`linear_lora` can compute ``u`` in its own launch (``shrink=True``):
    every module's A factors fit one pass (``n_modules * rank <= 128``) and lie evenly
    spaced in the cache (or there is one module)."""
    mods = list(modules)
    if len(mods) * rank > 128 or rank not in (16, 32, 64):
        return False
    d = mods[1] - mods[0] if len(mods) > 1 else 1
    return d > 0 and all(b - a == d for a, b in zip(mods, mods[1:]))


def lora_shrink_blocked(x: Tensor, u: Tensor, cache: FactorCache, segs: SegmentTable, modules,
                        status: Tensor | None = None) -> None:
    """:func:`lora_shrink` writing ``u`` (from :func:`blocked_u`) in the tile-blocked
    operand layout that :func:`linear_lora` stages with one bulk copy per tile."""
    dev = nat.require_cuda(x, u, segs.table)
    x2, ldx = _rows(x)
    T = x2.shape[0]
    if u.numel() < _blocked_elems(len(modules), T, segs.n_segs, cache.rank) or not u.is_contiguous():
        raise ValueError("u must be a contiguous blocked_u(n_modules, n_tokens, n_segs, rank) buffer")
    rc = nat.lib().lf_lora_shrink_blocked(
        nat.stream_ptr(dev), nat.dtype_code(x.dtype), x2.data_ptr(), ldx, T,
        cache.hidden, cache.rank, cache.a_ptr, cache.a_slot_stride, cache.a_module_stride,
        cache.n_slots, len(modules), nat.i32_array(modules), *_seg_args(segs),
        u.data_ptr(), nat.ptr(status))
    nat.check(rc, "lf_lora_shrink_blocked")


def linear_lora(x: Tensor, weight: Tensor | None, bias: Tensor | None, u: Tensor, cache: FactorCache,
                segs: SegmentTable, modules, module_cols: int, act: int = 0, out: Tensor | None = None,
                status: Tensor | None = None, shrink: bool = False, weight_t: Tensor | None = None) -> Tensor:
    """``act(x @ weight.T + bias + delta)`` on the tcgen05 GEMM with the LoRA delta in
    its accumulator: output columns ``[i * module_cols, (i + 1) * module_cols)`` get
    ``u[i] @ B(slot(t), modules[i])`` (``u`` from :func:`lora_shrink_blocked`).
    One rounding of the sum, where the reference rounds the projection and the delta
    apart; see ``lf_linear_lora``.  With ``shrink`` the same launch computes ``u`` first
    (``lf_linear_lora_shrink``; ``u`` is then an output, in the same blocked layout).
    ``weight_t``, the ``(K, N)`` transpose of ``weight`` (which may then be None), is
    read in the delta factors' operand form instead (``w_kn`` of the C entry points)."""
    dev = nat.require_cuda(x, weight, weight_t, bias, u, segs.table, out, status)
    x2, ldx = _rows(x)
    if weight_t is not None:
        K, N = weight_t.shape
        w, w_kn = (weight_t if weight_t.stride(-1) == 1 else weight_t.contiguous()), 1
    else:
        N, K = weight.shape
        w, w_kn = (weight if weight.stride(-1) == 1 else weight.contiguous()), 0
    if u.numel() < _blocked_elems(len(modules), x2.shape[0], segs.n_segs, cache.rank) or not u.is_contiguous() \
            or u.dtype != x.dtype:
        raise ValueError("u must be a contiguous blocked_u(n_modules, n_tokens, n_segs, rank) buffer of x's dtype")
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    o2 = out.reshape(-1, N)
    if o2.data_ptr() != out.data_ptr() or o2.stride(-1) != 1:
        raise ValueError("out must be viewable as rows without a copy")
    b = None if bias is None else (bias if bias.dtype == x.dtype else bias.to(x.dtype)).contiguous()
    if segs.n_tokens != x2.shape[0]:
        raise ValueError(f"segment table for {segs.n_tokens} tokens, x has {x2.shape[0]}")
    tp, pp = segs.pair_ptrs()
    if shrink:
        if cache.hidden != K:
            raise ValueError(f"the A factors take {cache.hidden} inputs, x has {K}")
        s_start, s_len, _, _, _, _ = segs.ptrs()
        rc = nat.lib().lf_linear_lora_shrink(
            nat.stream_ptr(dev), nat.dtype_code(x.dtype), x2.data_ptr(), ldx, w.data_ptr(), w.stride(0), w_kn,
            nat.ptr(b), o2.data_ptr(), o2.stride(0), x2.shape[0], N, K, int(act), u.data_ptr(), cache.rank,
            cache.a_ptr, cache.a_slot_stride, cache.a_module_stride, cache.b_ptr, cache.b_slot_stride,
            cache.b_module_stride, cache.n_slots, len(modules), nat.i32_array(modules), int(module_cols), s_start,
            s_len, segs.n_segs, tp, pp, nat.ptr(status))
        nat.check(rc, "lf_linear_lora_shrink")
        return out
    rc = nat.lib().lf_linear_lora(
        nat.stream_ptr(dev), nat.dtype_code(x.dtype), x2.data_ptr(), ldx, w.data_ptr(), w.stride(0), w_kn, nat.ptr(b),
        o2.data_ptr(), o2.stride(0), x2.shape[0], N, K, int(act), u.data_ptr(), cache.rank, cache.b_ptr,
        cache.b_slot_stride, cache.b_module_stride, cache.n_slots, len(modules), nat.i32_array(modules),
        int(module_cols), segs.n_segs, tp, pp, nat.ptr(status))
    nat.check(rc, "lf_linear_lora")
    return out


def lora_shrink(x: Tensor, u: Tensor, cache: FactorCache, segs: SegmentTable, modules,
                status: Tensor | None = None) -> None:
    """``u[m, t] = A_m(slot(t))^T x[t]`` rounded to the dtype; ``u`` is ``(n_mod, T, R)``."""
    dev = nat.require_cuda(x, u, segs.table)
    x2, ldx = _rows(x)
    rc = nat.lib().lf_lora_shrink(
        nat.stream_ptr(dev), nat.dtype_code(x.dtype), x2.data_ptr(), ldx, x2.shape[0],
        cache.hidden, cache.rank, cache.a_ptr, cache.a_slot_stride, cache.a_module_stride,
        cache.n_slots, len(modules), nat.i32_array(modules), *_seg_args(segs),
        u.data_ptr(), nat.ptr(status))
    nat.check(rc, "lf_lora_shrink")


def lora_expand(u: Tensor, y: Tensor, cache: FactorCache, segs: SegmentTable, modules, y_col_offsets,
                accumulate: bool, status: Tensor | None = None) -> None:
    """``y = [y +] round(u B)`` per op module (see :func:`lora_apply` for the column layout)."""
    dev = nat.require_cuda(u, y, segs.table)
    y2 = y.reshape(-1, y.shape[-1])
    if y2.data_ptr() != y.data_ptr() or y2.stride(-1) != 1:
        raise ValueError("y must be viewable as rows without a copy")
    rc = nat.lib().lf_lora_expand(
        nat.stream_ptr(dev), nat.dtype_code(y.dtype), u.data_ptr(), y2.data_ptr(), y2.stride(0),
        y2.shape[0], cache.hidden, cache.rank, cache.b_ptr, cache.b_slot_stride, cache.b_module_stride,
        cache.n_slots, len(modules), nat.i32_array(modules), nat.i64_array(y_col_offsets),
        *_seg_args(segs), 1 if accumulate else 0, nat.ptr(status))
    nat.check(rc, "lf_lora_expand")


def per_row_cache(a: Tensor, b: Tensor) -> FactorCache:
    """A factor cache over materialised per-row factors ``a (B,H,R)``, ``b (B,R,H)``:
    slot ``i`` is row ``i`` (what the reference's assemblers hand to ``LoraOps``)."""
    a = a.contiguous()
    b = b.contiguous()
    Bn, H, R = a.shape
    return FactorCache(a=a, b=b, a_offset=0, b_offset=0, a_slot_stride=H * R, b_slot_stride=R * H,
                       a_module_stride=0, b_module_stride=0, n_slots=Bn, hidden=H, rank=R)


class LoraOps:
    """Batched LoRA operations over buffers pre-allocated from the config.

    Same interface and contract as the reference's ``LoraOps``
    (``src/latefuse/ops/lora.py:7-80``): ``shrink(x, a_weights)`` fills ``out_A``
    ``(B, S, R)``, ``expand(b_weights)`` fills ``out_B`` ``(B, S, H)`` and ``output``
    returns it.  Both steps run the sm_100a kernels with row ``i`` of the batch
    using factor row ``i``; ``out_A`` is rounded to the model dtype exactly as the
    reference's ``bmm(..., out=_out_A)`` is.
    """

    def __init__(self, config: LoraServingConfig):
        B, S, H, R = config.batch_size, config.max_seq_len, config.hidden_size, config.lora_rank
        self._out_A = torch.empty(B, S, R, dtype=config.dtype, device=config.device)
        self._out_B = torch.empty(B, S, H, dtype=config.dtype, device=config.device)
        self._segs = SegmentTable.for_padded(list(range(B)), S, config.device)
        self._a: Tensor | None = None

    def shrink(self, x: Tensor, a_weights: Tensor) -> None:
        """First LoRA step: ``out_A = bmm(x, a_weights)``.

        Args:
            x:         (B, S, H) input hidden states
            a_weights: (B, H, R) stacked A matrices, one per sample
        """
        assert x.device == self._out_A.device, f"x on {x.device} but LoraOps buffers on {self._out_A.device}"
        assert a_weights.device == self._out_A.device, (
            f"a_weights on {a_weights.device} but buffers on {self._out_A.device}")
        B, S, R = self._out_A.shape
        H = self._out_B.shape[2]
        assert x.shape == (B, S, H), (
            f"x shape {tuple(x.shape)} != buffer shape {(B, S, H)}; "
            "LoraOps buffers are sized from config at init")
        assert a_weights.shape == (B, H, R), f"a_weights shape {tuple(a_weights.shape)} != expected {(B, H, R)}"
        a = a_weights.to(self._out_A.dtype).contiguous()
        self._a = a
        cache = FactorCache(a=a, b=a, a_offset=0, b_offset=0, a_slot_stride=H * R, b_slot_stride=R * H,
                            a_module_stride=0, b_module_stride=0, n_slots=B, hidden=H, rank=R)
        lora_shrink(x.to(self._out_A.dtype), self._out_A, cache, self._segs, [0])

    def expand(self, b_weights: Tensor) -> None:
        """Second LoRA step: ``out_B = bmm(out_A, b_weights)``; call ``shrink`` first.

        Args:
            b_weights: (B, R, H) stacked B matrices, one per sample
        """
        assert b_weights.device == self._out_B.device, (
            f"b_weights on {b_weights.device} but buffers on {self._out_B.device}")
        B, S, R = self._out_A.shape
        H = self._out_B.shape[2]
        assert b_weights.shape == (B, R, H), f"b_weights shape {tuple(b_weights.shape)} != expected {(B, R, H)}"
        b = b_weights.to(self._out_B.dtype).contiguous()
        cache = FactorCache(a=b, b=b, a_offset=0, b_offset=0, a_slot_stride=H * R, b_slot_stride=R * H,
                            a_module_stride=0, b_module_stride=0, n_slots=B, hidden=H, rank=R)
        lora_expand(self._out_A, self._out_B, cache, self._segs, [0], [0], accumulate=False)

    @property
    def output(self) -> Tensor:
        """The (B, S, H) LoRA delta from the last expand() call."""
        return self._out_B
