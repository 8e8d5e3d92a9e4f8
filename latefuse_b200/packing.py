"""Padding-free ("packed") batches for the native encoder.

A right-padded ``(B, S)`` batch with real lengths ``len_b`` holds ``sum(len_b)``
real tokens.  The reference runs every layer over all ``B*S`` positions and
keeps padded keys out of attention with the mask
(``src/latefuse/model/encoder.py:45-142``; the hf engine through HuggingFace's
attention mask).  No real token's output depends on a padded position: the
embeddings, projections, LoRA deltas, LayerNorms and FFN are per token, and
attention never reads a padded key.  So the native encoder can run the per-token
ops on the real tokens only and attention per sequence (``cu_seqlens``), with
the same results on every real token.

Rows are laid out sorted by adapter slot (stable), so all rows of one tenant
are adjacent and the LoRA delta sees one segment per tenant run rather than one
per row.  Everything the device needs (the attention work list, token ids,
position ids, token types, ``cu_seqlens``, the first token of each row, the row
of each token, row lengths) goes over in one pinned host-to-device copy.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import Tensor

from latefuse_b200.lora import SegmentTable


@dataclass
class PackedBatch:
    """One mixed-tenant batch with its padding removed.

    Packed order is the rows sorted by slot; ``order[i]`` is the input row at
    packed position ``i``.  Device tensors are int32 views of one buffer.
    """

    n_rows: int
    n_tokens: int
    max_len: int
    lengths: list[int]          # per input row
    order: list[int]            # packed position -> input row
    slots: list[int]            # per input row
    ids: Tensor                 # (n_tokens,) token ids
    positions: Tensor           # (n_tokens,) position ids
    token_types: Tensor         # (n_tokens,) token type ids
    cu_seqlens: Tensor          # (n_rows + 1,) sequence boundaries in packed order
    first_token: Tensor         # (n_rows,) packed index of each input row's first token
    row_of_token: Tensor        # (n_tokens,) input row of each packed token
    row_lengths: Tensor         # (n_rows,) per input row
    segments: SegmentTable      # LoRA segments: runs of rows with one slot
    attn_items: Tensor          # (n_attn_items, 4) {row_start, len, q_tile, 0}, longest sequences first
    host_bytes: int             # bytes copied host -> device for this batch


def attention_items(starts, lengths) -> np.ndarray:
    """The attention work list of packed sequences: ``(n, 4)`` int64 records
    ``{row_start, len, q_tile, 0}``, one per (sequence, 128-query tile), the
    sequences with more key tiles first so that the persistent kernel's
    round-robin over CTAs balances."""
    starts = np.asarray(starts, dtype=np.int64)
    lengths = np.asarray(lengths, dtype=np.int64)
    n_qt = (lengths + 127) // 128
    seq_order = np.argsort(-n_qt, kind="stable")
    reps = n_qt[seq_order]
    total = int(reps.sum())
    items = np.zeros((total, 4), dtype=np.int64)
    items[:, 0] = np.repeat(starts[seq_order], reps)
    items[:, 1] = np.repeat(lengths[seq_order], reps)
    items[:, 2] = np.arange(total) - np.repeat(np.cumsum(reps) - reps, reps)
    return items


def pack_rows(input_ids: Tensor, lengths: list[int], slots: list[int], position_pad: int | None,
              token_type_ids: Tensor | None, device: torch.device) -> PackedBatch:
    """Pack the real tokens of right-padded host rows (``1 <= lengths[b] <= S``).

    Position ids follow the model's rule on the padded rows, so packing changes
    no position: ``position_pad=None`` numbers every row ``0, 1, 2 ...`` (BERT);
    an integer ``pad`` numbers the non-pad tokens of a row ``pad+1, pad+2 ...``
    and gives pad tokens ``pad`` (the RoBERTa family, from ``input_ids != pad``).
    """
    B, S = input_ids.shape
    if len(lengths) != B or len(slots) != B:
        raise ValueError(f"{B} rows but {len(lengths)} lengths and {len(slots)} slots")
    lens = np.asarray(lengths, dtype=np.int64)
    if B == 0 or lens.min() < 1 or lens.max() > S:
        raise ValueError("every packed row needs 1..S real tokens")
    order = sorted(range(B), key=lambda b: slots[b])  # stable: ties keep input order
    olens = lens[order]
    cu = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(olens, out=cu[1:])
    T = int(cu[-1])
    # flat (row * S + col) index of every real token, in packed order
    row_base = np.repeat(np.asarray(order, dtype=np.int64) * S, olens)
    col = np.arange(T, dtype=np.int64) - np.repeat(cu[:-1], olens)
    sel = row_base + col
    first = np.empty(B, dtype=np.int64)
    first[order] = cu[:-1]

    items = attention_items(cu[:-1], olens)
    n_items = items.shape[0]

    n_parts = 4 * n_items + 3 * T + (B + 1) + B + T + B
    buf = torch.empty(n_parts, dtype=torch.int32, pin_memory=device.type == "cuda")
    a = buf.numpy()
    a[:4 * n_items] = items.reshape(-1)
    o = 4 * n_items
    ids_sel = input_ids.reshape(-1).numpy()[sel]
    a[o:o + T] = ids_sel
    o += T
    if position_pad is None:
        a[o:o + T] = col
    else:
        # within a row the real tokens are a prefix, so a running count over the
        # packed tokens restarted at each row gives the padded rows' cumsum
        ne = (ids_sel != position_pad).astype(np.int64)
        cs = np.cumsum(ne)
        base = np.repeat(cs[cu[:-1]] - ne[cu[:-1]], olens)
        a[o:o + T] = (cs - base) * ne + position_pad
    o += T
    a[o:o + T] = token_type_ids.reshape(-1).numpy()[sel] if token_type_ids is not None else 0
    o += T
    a[o:o + B + 1] = cu
    o += B + 1
    a[o:o + B] = first
    o += B
    a[o:o + T] = np.repeat(np.asarray(order, dtype=np.int64), olens)
    o += T
    a[o:o + B] = lens
    dev_buf = buf.to(device, non_blocking=True) if device.type == "cuda" else buf.clone()
    views, o = [dev_buf[:4 * n_items].view(n_items, 4)], 4 * n_items
    for n in (T, T, T, B + 1, B, T, B):
        views.append(dev_buf[o:o + n])
        o += n

    # LoRA segments: maximal runs of packed rows that share a slot
    starts, seg_lens, seg_slots = [], [], []
    for i, b in enumerate(order):
        if seg_slots and seg_slots[-1] == slots[b]:
            seg_lens[-1] += int(lens[b])
        else:
            starts.append(int(cu[i]))
            seg_lens.append(int(lens[b]))
            seg_slots.append(int(slots[b]))
    segs = SegmentTable(starts, seg_lens, seg_slots, T, device)
    return PackedBatch(n_rows=B, n_tokens=T, max_len=int(lens.max()), lengths=[int(n) for n in lens],
                       order=order, slots=list(slots), ids=views[1], positions=views[2], token_types=views[3],
                       cu_seqlens=views[4], first_token=views[5], row_of_token=views[6], row_lengths=views[7],
                       segments=segs, attn_items=views[0], host_bytes=n_parts * 4 + segs.host.numel() * 4)
