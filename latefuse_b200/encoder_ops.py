"""The encoder's elementwise ops on the native kernels.

``linear`` is ``nn.Linear`` (with the FFN's GELU fused when asked) on this
library's tcgen05 GEMM; ``add_layernorm`` is ``nn.LayerNorm(sublayer_out + residual)`` in one pass over
HBM (``src/latefuse/model/encoder.py:137,141``; with no residual, the embeddings'
LayerNorm at ``:275``), ``gelu`` is the exact erf GELU of the FFN (``:122,139``),
both with torch's rounding points, and ``attention_varlen`` is the encoder's
masked self-attention (``:82-98``) on a padding-free batch (see the
``lf_*`` declarations in ``include/latefuse_b200.h``).
"""

from __future__ import annotations

import torch
from torch import Tensor

from latefuse_b200 import _native as nat


def _rows(t: Tensor) -> tuple[Tensor, int]:
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2, t2.stride(0)


def add_layernorm(a: Tensor, b: Tensor | None, weight: Tensor, bias: Tensor, eps: float,
                  out: Tensor | None = None, vec: Tensor | None = None) -> Tensor:
    """``layer_norm(a + b)`` (``b`` may be None) over the last dimension; or, with
    ``vec`` (one row, e.g. a projection bias) instead of ``b``, ``layer_norm(a + vec)``."""
    dev = nat.require_cuda(a, b, weight, bias, out, vec)
    H = a.shape[-1]
    a2, lda = _rows(a)
    b2, ldb = _rows(b) if b is not None else (None, 0)
    if out is None:
        out = torch.empty(a.shape, dtype=a.dtype, device=a.device)
    o2, ldo = _rows(out)
    w = weight if weight.dtype == a.dtype else weight.to(a.dtype)
    bb = bias if bias.dtype == a.dtype else bias.to(a.dtype)
    v = None if vec is None else (vec if vec.dtype == a.dtype else vec.to(a.dtype)).contiguous()
    rc = nat.lib().lf_add_layernorm(nat.stream_ptr(dev), nat.dtype_code(a.dtype), a2.data_ptr(), lda,
                                    nat.ptr(b2), ldb, nat.ptr(v), w.contiguous().data_ptr(),
                                    bb.contiguous().data_ptr(), float(eps), a2.shape[0], H, o2.data_ptr(), ldo)
    nat.check(rc, "lf_add_layernorm")
    return out


def embed_layernorm(ids: Tensor, positions: Tensor, types: Tensor | None, word: Tensor, pos: Tensor,
                    type_: Tensor, weight: Tensor, bias: Tensor, eps: float, status: Tensor | None = None) -> Tensor:
    """``layer_norm((word[ids] + type_[types]) + pos[positions])`` for int32 index vectors
    (each sum rounded to the tables' dtype, as torch's embedding adds are), one native
    launch.  ``types`` None takes type row 0 everywhere.  Returns ``(len(ids), H)``."""
    dev = nat.require_cuda(ids, positions, types, word, pos, type_, weight, bias, status)
    for t in (ids, positions, types):
        if t is not None and (t.dtype != torch.int32 or not t.is_contiguous()):
            raise ValueError("ids, positions and types must be contiguous int32 tensors")
    n, H = ids.shape[0], word.shape[1]
    if positions.shape[0] != n or (types is not None and types.shape[0] != n):
        raise ValueError(f"{n} ids but {positions.shape[0]} positions")
    out = torch.empty(n, H, dtype=word.dtype, device=word.device)
    w = weight if weight.dtype == word.dtype else weight.to(word.dtype)
    bb = bias if bias.dtype == word.dtype else bias.to(word.dtype)
    rc = nat.lib().lf_embed_layernorm(
        nat.stream_ptr(dev), nat.dtype_code(word.dtype), word.data_ptr(), word.stride(0), word.shape[0],
        ids.data_ptr(), pos.data_ptr(), pos.stride(0), pos.shape[0], positions.data_ptr(), type_.data_ptr(),
        type_.stride(0), type_.shape[0], nat.ptr(types), w.contiguous().data_ptr(), bb.contiguous().data_ptr(),
        float(eps), n, H, out.data_ptr(), out.stride(0), nat.ptr(status))
    nat.check(rc, "lf_embed_layernorm")
    return out


def gelu(x: Tensor, out: Tensor | None = None) -> Tensor:
    """Exact (erf) GELU of a contiguous tensor."""
    dev = nat.require_cuda(x, out)
    if not x.is_contiguous():
        x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    rc = nat.lib().lf_gelu(nat.stream_ptr(dev), nat.dtype_code(x.dtype), x.data_ptr(), out.data_ptr(), x.numel())
    nat.check(rc, "lf_gelu")
    return out


def attention_varlen(qkv: Tensor, n_heads: int, items: Tensor, scale: float, out: Tensor | None = None,
                     status: Tensor | None = None) -> Tensor:
    """Self-attention of packed sequences, head_dim 64, read straight from the fused
    ``(T, 3H)`` projection output (q, k, v at columns 0, H, 2H); ``items`` is the
    ``(n, 4)`` device int32 work list of :class:`~latefuse_b200.packing.PackedBatch`.
    Returns ``(T, H)``."""
    dev = nat.require_cuda(qkv, items, out, status)
    if items.dtype != torch.int32 or items.dim() != 2 or items.shape[1] != 4 or not items.is_contiguous():
        raise ValueError("items must be a contiguous (n, 4) int32 tensor (PackedBatch.attn_items)")
    T, W = qkv.shape
    H = W // 3
    if qkv.stride(-1) != 1:
        raise ValueError("qkv rows must be contiguous")
    if out is None:
        out = torch.empty(T, H, dtype=qkv.dtype, device=qkv.device)
    elif out.dtype != qkv.dtype or out.shape != (T, H) or out.stride(-1) != 1:
        raise ValueError(f"out must be a ({T}, {H}) {qkv.dtype} tensor with contiguous rows")
    rc = nat.lib().lf_attention_varlen(nat.stream_ptr(dev), nat.dtype_code(qkv.dtype), qkv.data_ptr(), qkv.stride(0),
                                       T, 0, H, 2 * H, n_heads, H // n_heads, items.data_ptr(), items.shape[0],
                                       float(scale), out.data_ptr(), out.stride(0), nat.ptr(status))
    nat.check(rc, "lf_attention_varlen")
    return out


ACT_NONE, ACT_GELU = 0, 1


def linear(x: Tensor, weight: Tensor, bias: Tensor | None, act: int = ACT_NONE,
           out: Tensor | None = None) -> Tensor:
    """``act(x @ weight.T + bias)`` (``act``: ``ACT_NONE`` or ``ACT_GELU``, the exact erf
    GELU) for bf16/f16 ``x (..., K)`` and an ``nn.Linear`` weight ``(N, K)``;
    N % 256 == 0, K % 64 == 0.  ``out`` must be viewable as rows without a copy."""
    dev = nat.require_cuda(x, weight, bias, out)
    x2, ldx = _rows(x)
    N, K = weight.shape
    if x2.shape[1] != K:
        raise ValueError(f"x has {x2.shape[1]} columns, weight expects {K}")
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    o2 = out.reshape(-1, N)
    if o2.data_ptr() != out.data_ptr() or o2.stride(-1) != 1 or (out.dim() > 2 and not out.is_contiguous()):
        raise ValueError("out must be viewable as rows without a copy")
    b = None if bias is None else (bias if bias.dtype == x.dtype else bias.to(x.dtype)).contiguous()
    rc = nat.lib().lf_linear(nat.stream_ptr(dev), nat.dtype_code(x.dtype), x2.data_ptr(), ldx, w.data_ptr(),
                             w.stride(0), nat.ptr(b), o2.data_ptr(), o2.stride(0), x2.shape[0], N, K, int(act), None)
    nat.check(rc, "lf_linear")
    return out


def linear_accumulate(x: Tensor, weight: Tensor, y: Tensor, bias: Tensor | None = None) -> Tensor:
    """``y += x @ weight.T (+ bias)`` in place, summed in f32 and rounded once (cuBLAS's
    ``addmm_`` with beta = 1) for bf16/f16 ``x (..., K)``, an ``nn.Linear`` weight
    ``(N, K)`` and ``y (..., N)`` viewable as rows without a copy; N % 256 == 0,
    K % 64 == 0.  Returns ``y``."""
    dev = nat.require_cuda(x, weight, y, bias)
    x2, ldx = _rows(x)
    N, K = weight.shape
    if x2.shape[1] != K:
        raise ValueError(f"x has {x2.shape[1]} columns, weight expects {K}")
    if y.dtype != x.dtype:
        raise ValueError(f"y is {y.dtype}, x is {x.dtype}")
    y2 = y.reshape(-1, N)
    if y2.data_ptr() != y.data_ptr() or y2.stride(-1) != 1 or (y.dim() > 2 and not y.is_contiguous()) or \
            y2.shape[0] != x2.shape[0]:
        raise ValueError(f"y must be ({x2.shape[0]}, {N}) rows viewable without a copy")
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    b = None if bias is None else (bias if bias.dtype == x.dtype else bias.to(x.dtype)).contiguous()
    rc = nat.lib().lf_linear_accumulate(nat.stream_ptr(dev), nat.dtype_code(x.dtype), x2.data_ptr(), ldx,
                                        w.data_ptr(), w.stride(0), nat.ptr(b), y2.data_ptr(), y2.stride(0),
                                        x2.shape[0], N, K, None)
    nat.check(rc, "lf_linear_accumulate")
    return y
