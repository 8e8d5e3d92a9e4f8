"""Oracle for pooling, normalisation and per-tenant heads (CPU, PyTorch)."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor


def pool_tokens(hidden: Tensor, mask: Tensor | None, strategy: str) -> Tensor:
    """``src/latefuse/ops/pooling.py:36-73``: CLS row, or the mask-weighted mean with the
    count clamped at 1e-9 (computed in the hidden states' dtype)."""
    if strategy == "cls":
        return hidden[:, 0]
    if strategy == "mean":
        if mask is None:
            return hidden.mean(dim=1)
        m = mask.unsqueeze(-1).to(hidden.dtype)
        summed = (hidden * m).sum(dim=1)
        counts = m.sum(dim=1).clamp(min=1e-9)
        return summed / counts
    raise ValueError(f"unknown pooling strategy {strategy!r}")


def normalize(x: Tensor) -> Tensor:
    """``F.normalize(p=2, dim=-1)`` (``src/latefuse/tasks/embedding.py:69-70``)."""
    return F.normalize(x, p=2, dim=-1)


def assemble_heads(heads: dict, tenants: list[str], H: int, dtype) -> tuple[Tensor, Tensor, list[int]]:
    """Zero-padded ``(B, max_labels, H)`` coef / ``(B, max_labels)`` intercept
    (``src/latefuse/tasks/heads.py:125-158``); ``heads[t] = (coef (n,H), intercept (n,))``."""
    num_labels = [heads[t][0].shape[0] for t in tenants]
    L = max(num_labels)
    coef = torch.zeros(len(tenants), L, H, dtype=dtype)
    icpt = torch.zeros(len(tenants), L, dtype=dtype)
    for i, t in enumerate(tenants):
        c, b = heads[t]
        coef[i, : c.shape[0]] = c.to(dtype)
        icpt[i, : c.shape[0]] = b.to(dtype)
    return coef, icpt, num_labels


def head_logits(pooled: Tensor, coef: Tensor, intercept: Tensor) -> Tensor:
    """``bmm(pooled (B,1,H), coef^T) + intercept`` in the model dtype (``src/latefuse/ops/head.py:50-51``):
    the dot product is stored in the dtype, then the intercept is added in the dtype."""
    dt = pooled.dtype
    dots = torch.bmm(pooled.float().unsqueeze(1), coef.float().transpose(1, 2)).to(dt)
    return (dots.float() + intercept.float().unsqueeze(1)).to(dt)[:, 0]


def softmax(row: list[float]) -> list[float]:
    """Max-shifted softmax in Python floats (``src/latefuse/tasks/classification.py:109-115``)."""
    top = max(row)
    exps = [math.exp(v - top) for v in row]
    total = sum(exps)
    return [e / total for e in exps]


def sigmoid(row: list[float]) -> list[float]:
    """``src/latefuse/tasks/classification.py:118-119``."""
    return [1.0 / (1.0 + math.exp(-row[0]))]


def ragged(scores: Tensor, num_labels: list[int]) -> list[list[float]]:
    """Per-row ``scores[i, :n].tolist()`` (``src/latefuse/tasks/classification.py:67-70``)."""
    return [scores[i, :n].tolist() for i, n in enumerate(num_labels)]


def probabilities(logits: list[list[float]]) -> list[list[float]]:
    """Sigmoid for one-logit rows, softmax otherwise (``classification.py:81-84``)."""
    return [sigmoid(r) if len(r) == 1 else softmax(r) for r in logits]


def predictions(logits: list[list[float]]) -> list[int]:
    """Argmax (first on ties) or ``logit > 0`` for one-logit rows (``classification.py:86-98``)."""
    out = []
    for row in logits:
        out.append(int(row[0] > 0.0) if len(row) == 1 else max(range(len(row)), key=row.__getitem__))
    return out
