"""Oracle for the LoRA delta and the batch gather (CPU, PyTorch).

Reference arithmetic (``src/latefuse/ops/lora.py:57,75`` and the hook
``src/latefuse/model/hf_wrapper.py:213-217``)::

    out_A = bmm(x, A_batched)          # (B,S,H)x(B,H,R), result stored in the model dtype
    out_B = bmm(out_A, B_batched)      # (B,S,R)x(B,R,H), result stored in the model dtype
    y     = output + out_B             # add in the model dtype

The functions below reproduce those three rounding points explicitly with f32
accumulation (``round(...)`` = cast to the model dtype).
"""

from __future__ import annotations

import torch
from torch import Tensor


def _rnd(t: Tensor, dtype: torch.dtype) -> Tensor:
    return t.to(dtype).to(torch.float32)


def lora_delta(x: Tensor, a: Tensor, b: Tensor) -> Tensor:
    """``round(round(x @ a) @ b)`` per batch row: x ``(B,S,H)``, a ``(B,H,R)``, b ``(B,R,H)``.

    Follows ``LoraOps.shrink`` / ``expand`` (``src/latefuse/ops/lora.py:29-75``).
    Returns the delta in the model dtype.
    """
    dt = x.dtype
    u = _rnd(torch.bmm(x.float(), a.float()), dt)
    return torch.bmm(u, b.float()).to(dt)


def lora_delta_loop(x: Tensor, a: Tensor, b: Tensor) -> Tensor:
    """Per-sample loop form (``tests/test_ops.py:56``): ``stack([x[i] @ a[i] @ b[i]])``."""
    return torch.stack([x[i] @ a[i] @ b[i] for i in range(x.shape[0])])


def hook_output(output: Tensor, x: Tensor, a: Tensor, b: Tensor) -> Tensor:
    """``output + delta`` in the model dtype (``src/latefuse/model/hf_wrapper.py:215-217``)."""
    d = lora_delta(x, a, b)
    return (output.float() + d.float()).to(output.dtype)


def segmented_apply(x: Tensor, y: Tensor, a_of, b_of, segments, col_offsets=(0,), modules=(0,),
                    accumulate: bool = True) -> Tensor:
    """Token-row form over a segment table: returns a new ``y``.

    x ``(T,H)``; y ``(T,C)``; ``segments`` = iterable of (start, length, slot);
    ``a_of(slot, module)`` -> ``(H,R)``, ``b_of(slot, module)`` -> ``(R,H)``.
    Rows covered by a segment get the reference arithmetic above with that
    slot's factors; other rows get a zero delta.
    """
    dt = x.dtype
    H = x.shape[1]
    out = y.clone()
    if not accumulate:
        for off in col_offsets:
            out[:, off : off + H] = 0
    for (start, length, slot) in segments:
        if length <= 0:
            continue
        rows = slice(start, start + length)
        xs = x[rows].float()
        for m, off in zip(modules, col_offsets):
            u = _rnd(xs @ a_of(slot, m).float(), dt)
            d = _rnd(u @ b_of(slot, m).float(), dt)
            cur = y[rows, off : off + H].float() if accumulate else torch.zeros_like(d)
            out[rows, off : off + H] = (cur + d).to(dt)
    return out


def index_select_gather(packed: Tensor, row_of: dict, ids) -> Tensor:
    """``packed.index_select(0, [row_of[i] for i in ids])`` (``src/latefuse/weights/batch.py:172-203``)."""
    idx = torch.tensor([row_of[i] for i in ids], dtype=torch.long)
    return packed.index_select(0, idx)


def cpu_assemble(wa_of, ids, layer: int) -> Tensor:
    """The CPU assembler's per-layer stack (``src/latefuse/weights/batch.py:64-69`` + engine cat)."""
    return torch.cat([wa_of(i)[layer].unsqueeze(0) for i in ids], dim=0)
