"""Pooling, normalisation and per-tenant heads on the GPU.

Mirrors ``src/latefuse/ops/pooling.py`` (``POOLING_STRATEGIES``,
``validate_pooling``, ``pool_tokens``) and ``src/latefuse/ops/head.py``
(``LRHeadOps.predict_proba``); all of them run the one native kernel
``lf_head_forward`` (pool -> L2 norm -> gather-GEMV over packed heads -> masked
softmax/sigmoid).
"""

from __future__ import annotations

import torch
from torch import Tensor

from latefuse_b200 import _native as nat

#: Accepted ``pooling=`` values. ``"auto"`` defers to the engine.
POOLING_STRATEGIES = ("auto", "cls", "mean")


def validate_pooling(strategy: str) -> str:
    """Return ``strategy`` if known, else raise naming the alternatives."""
    if strategy not in POOLING_STRATEGIES:
        raise ValueError(
            f"unknown pooling strategy {strategy!r}; expected one of {', '.join(map(repr, POOLING_STRATEGIES))}"
        )
    return strategy


def _mask_i64(mask: Tensor | None) -> Tensor | None:
    if mask is None:
        return None
    if mask.dtype != torch.int64:
        mask = mask.to(torch.int64)
    return mask.contiguous()


def head_forward(hidden: Tensor, *, pooling: str, mask: Tensor | None = None, pooled_out: Tensor | None = None,
                 normed_out: Tensor | None = None, coef: Tensor | None = None, bias: Tensor | None = None,
                 head_table: Tensor | None = None, n_max: int = 0, logits_out: Tensor | None = None,
                 probs_out: Tensor | None = None, status: Tensor | None = None) -> None:
    """Run ``lf_head_forward`` on the current stream.

    ``hidden`` is ``(B, S, H)`` for ``pooling in {"cls", "mean"}`` or ``(B, H)`` for
    ``"none"``; ``head_table`` is the ``(2, B)`` int32 (offset, num_labels) table.
    """
    dev = nat.require_cuda(hidden, mask, pooled_out, normed_out, coef, bias, head_table, logits_out, probs_out)
    if hidden.stride(-1) != 1:
        hidden = hidden.contiguous()
    if pooling == "none":
        B, H = hidden.shape
        S, ld_b, ld_s = 1, hidden.stride(0), 0
    else:
        B, S, H = hidden.shape
        ld_b, ld_s = hidden.stride(0), hidden.stride(1)
    mask = _mask_i64(mask)
    off_ptr = n_ptr = None
    if head_table is not None:
        off_ptr = head_table.data_ptr()
        n_ptr = off_ptr + head_table.stride(0) * 4
    rc = nat.lib().lf_head_forward(
        nat.stream_ptr(dev), nat.dtype_code(hidden.dtype), hidden.data_ptr(), ld_b, ld_s, nat.ptr(mask),
        B, S, H, nat.LF_POOL[pooling], nat.ptr(pooled_out), nat.ptr(normed_out), nat.ptr(coef), nat.ptr(bias),
        coef.shape[0] if coef is not None else 0, off_ptr, n_ptr, n_max, nat.ptr(logits_out),
        nat.ptr(probs_out), nat.ptr(status))
    nat.check(rc, "lf_head_forward")


def head_forward_rows(hidden: Tensor, row_index: Tensor | None, *, pooler_w: Tensor | None = None,
                      pooler_b: Tensor | None = None, pooled_out: Tensor | None = None,
                      normed_out: Tensor | None = None, coef: Tensor | None = None, bias: Tensor | None = None,
                      head_table: Tensor | None = None, n_max: int = 0, logits_out: Tensor | None = None,
                      probs_out: Tensor | None = None, status: Tensor | None = None) -> None:
    """Run ``lf_head_forward_rows`` on the current stream: rows ``row_index`` (int32,
    ``(B,)``) of the packed ``(n_tokens, H)`` ``hidden``, optionally through the
    pooler ``tanh(pooler_w x + pooler_b)`` (then ``pooled_out`` is required), then
    the L2 norm / per-tenant head / softmax of :func:`head_forward`."""
    dev = nat.require_cuda(hidden, row_index, pooler_w, pooler_b, pooled_out, normed_out, coef, bias, head_table,
                           logits_out, probs_out)
    if hidden.dim() != 2 or hidden.stride(-1) != 1:
        raise ValueError("head_forward_rows: hidden must be (n_tokens, H) with unit column stride")
    T, H = hidden.shape
    if row_index is not None:
        if row_index.dtype != torch.int32 or not row_index.is_contiguous():
            raise ValueError("head_forward_rows: row_index must be a contiguous int32 tensor")
        B = row_index.numel()
    else:
        B = T
    if pooler_w is not None:
        if pooled_out is None:
            raise ValueError("head_forward_rows: the pooler writes its rows to pooled_out")
        if tuple(pooler_w.shape) != (H, H) or not pooler_w.is_contiguous():
            raise ValueError(f"head_forward_rows: pooler_w must be a contiguous ({H}, {H}) tensor")
    for name, t in (("pooled_out", pooled_out), ("normed_out", normed_out)):
        if t is not None and (tuple(t.shape) != (B, H) or not t.is_contiguous()):
            raise ValueError(f"head_forward_rows: {name} must be a contiguous ({B}, {H}) tensor")
    off_ptr = n_ptr = None
    if head_table is not None:
        off_ptr = head_table.data_ptr()
        n_ptr = off_ptr + head_table.stride(0) * 4
    rc = nat.lib().lf_head_forward_rows(
        nat.stream_ptr(dev), nat.dtype_code(hidden.dtype), hidden.data_ptr(), hidden.stride(0), nat.ptr(row_index),
        B, H, nat.ptr(pooler_w), nat.ptr(pooler_b), nat.ptr(pooled_out), nat.ptr(normed_out), nat.ptr(coef),
        nat.ptr(bias), coef.shape[0] if coef is not None else 0, off_ptr, n_ptr, n_max, nat.ptr(logits_out),
        nat.ptr(probs_out), nat.ptr(status))
    nat.check(rc, "lf_head_forward_rows")


def pool_tokens(hidden_states: Tensor, attention_mask: Tensor | None, strategy: str) -> Tensor:
    """Reduce ``(B, S, H)`` to ``(B, H)`` under ``"cls"`` or ``"mean"`` (native kernel).

    ``"mean"`` is the mask-weighted mean with the count clamped at 1e-9, as in the
    reference (``src/latefuse/ops/pooling.py:36-73``).  ``"auto"`` is rejected:
    it names an engine-specific pooler that the engine must resolve.
    """
    if strategy == "auto":
        raise ValueError(
            "pooling='auto' must be resolved by the engine before pooling; pass 'cls' or 'mean' to pool_tokens()"
        )
    if strategy not in ("cls", "mean"):
        raise ValueError(f"unknown pooling strategy {strategy!r}")
    B, _, H = hidden_states.shape
    out = torch.empty(B, H, dtype=hidden_states.dtype, device=hidden_states.device)
    head_forward(hidden_states, pooling=strategy, mask=attention_mask if strategy == "mean" else None,
                 pooled_out=out)
    return out


def l2_normalize(x: Tensor) -> Tensor:
    """``F.normalize(x, p=2, dim=-1)`` for ``(B, H)`` rows, on the native kernel."""
    out = torch.empty_like(x)
    head_forward(x, pooling="none", normed_out=out)
    return out


class LRHeadOps:
    """Batched logistic-regression inference for a mixed-tenant batch.

    Same contract as the reference (``src/latefuse/ops/head.py:15-52``): fills
    ``out (B, 1, max_labels)`` with ``pooled . coef^T + intercept`` where
    ``coef (B, max_labels, H)`` / ``intercept (B, max_labels)`` are zero-padded.
    """

    @staticmethod
    def predict_proba(pooled: Tensor, coef: Tensor, intercept: Tensor, out: Tensor) -> Tensor:
        assert coef.device == pooled.device, f"pooled on {pooled.device} but coef on {coef.device}"
        assert intercept.device == pooled.device, f"pooled on {pooled.device} but intercept on {intercept.device}"
        assert out.device == pooled.device, f"pooled on {pooled.device} but out on {out.device}"
        B, L, H = coef.shape
        table = torch.tensor([[b * L for b in range(B)], [L] * B], dtype=torch.int32, device=pooled.device)
        logits = torch.empty(B, L, dtype=coef.dtype, device=pooled.device)
        head_forward(pooled.reshape(B, H), pooling="none", coef=coef.reshape(B * L, H).contiguous(),
                     bias=intercept.reshape(B * L).contiguous(), head_table=table, n_max=L, logits_out=logits)
        out.copy_(logits.view(B, 1, L))
        return out
