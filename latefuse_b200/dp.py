"""Data-parallel serving over the GPUs of one box.

Rows (sequences) are independent given a replicated frozen base and a
replicated adapter cache, so a mixed-tenant global batch is split across ranks
(one process per GPU) with no exchange during the forward; the only collective
is one all-gather of the per-row outputs (embeddings or logits) at the end.
The reference has no multi-GPU path at all (its scale-out is independent
replicas behind a router, ``deploy/server/routing.py:1-12``).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
import torch.distributed as dist
from torch import Tensor


def _lpt(costs: Sequence[float], world: int, cap: list[int] | None) -> list[list[int]]:
    """Longest-processing-time greedy: rows in decreasing cost, each to the rank with
    the least load so far (and room under ``cap``, when given); ties to the lower rank."""
    if world <= 0:
        raise ValueError("world must be positive")
    parts: list[list[int]] = [[] for _ in range(world)]
    load = [0.0] * world
    for i in sorted(range(len(costs)), key=lambda k: (-float(costs[k]), k)):
        ranks = range(world) if cap is None else [k for k in range(world) if len(parts[k]) < cap[k]]
        r = min(ranks, key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += float(costs[i])
    return [sorted(p) for p in parts]


def partition_rows(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Assign rows to ``world`` ranks for the padded forward, whose cost is the same
    for every row: equal row counts (+-1), and within that the real tokens balanced.
    Each rank's rows are returned in input order."""
    n = len(lengths)
    cap = [n // max(world, 1) + (1 if r < n % max(world, 1) else 0) for r in range(max(world, 1))]
    return _lpt([int(x) for x in lengths], world, cap)


#: tokens of context at which one token's attention costs as much time as its
#: projections and FFN (the packed bge-m3-shaped forward: attention is about a
#: sixth of the step at a mean length of 272)
ATTENTION_TOKENS = 1430.0


def packed_cost(length: int, attention_tokens: float = ATTENTION_TOKENS) -> float:
    """Relative time of one row in the padding-free forward: per-token work (the
    projections, FFN and LoRA) plus attention, which grows with the row's length."""
    return float(length) * (1.0 + float(length) / attention_tokens)


def partition_tokens(lengths: Sequence[int], world: int,
                     attention_tokens: float = ATTENTION_TOKENS) -> list[list[int]]:
    """Assign rows to ``world`` ranks for the padding-free forward, whose cost follows
    each row's real length (:func:`packed_cost`), not the row count: row counts may
    differ between ranks.  Each rank's rows are returned in input order."""
    return _lpt([packed_cost(int(x), attention_tokens) for x in lengths], world, None)


def all_gather_rows(local: Tensor, counts: Sequence[int], group=None) -> Tensor:
    """Concatenate every rank's ``(counts[r], ...)`` rows in rank order.

    Rows are padded to the largest count for the collective (one
    ``all_gather_into_tensor`` over NCCL; the list form on other backends).
    """
    world = dist.get_world_size(group)
    mx = max(counts)
    pad = local.new_zeros((mx,) + tuple(local.shape[1:]))
    pad[: local.shape[0]] = local
    if dist.get_backend(group) == "nccl":
        out = local.new_empty((world * mx,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, pad, group=group)
        chunks = out.split(mx)
    else:
        chunks = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(chunks, pad, group=group)
    return torch.cat([c[:k] for c, k in zip(chunks, counts)], 0)


class DataParallelEmbedder:
    """Runs one :class:`~latefuse_b200.tasks.MultiTenantEmbedder` per rank over a shard
    of each global batch and returns the full result, in input order, on every rank."""

    def __init__(self, embedder, group=None):
        self.embedder = embedder
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def partition(self, lengths: Sequence[int]) -> list[list[int]]:
        """Rows of each rank: balanced on packed cost when the embedder runs the
        padding-free forward, on row count (then tokens) otherwise."""
        model = getattr(self.embedder, "model", None)
        packed = getattr(self.embedder, "pack_tokens", False) and getattr(model, "supports_packing", False)
        return partition_tokens(lengths, self.world) if packed else partition_rows(lengths, self.world)

    def embed_tokens(self, input_ids: Tensor, attention_mask: Tensor, tenants: Sequence[str], **kw) -> Tensor:
        """Embed a global pre-tokenized batch (host tensors; every rank passes the same batch)."""
        lengths = attention_mask.sum(1).tolist()
        parts = self.partition(lengths)
        mine = parts[self.rank]
        idx = torch.tensor(mine, dtype=torch.long)
        local = self.embedder.embed_tokens(input_ids[idx], attention_mask[idx], [tenants[i] for i in mine], **kw)
        rows = all_gather_rows(local, [len(p) for p in parts], self.group)
        order = torch.tensor([i for p in parts for i in p], dtype=torch.long, device=rows.device)
        out = torch.empty_like(rows)
        out[order] = rows
        return out

    def embed_tokens_stream(self, batches, *, depth: int = 2, **kw):
        """:meth:`embed_tokens` over an iterable of global ``(input_ids, attention_mask,
        tenants)`` batches with up to ``depth`` in flight; yields each full result as a
        pinned host tensor, in order (every rank the same)."""
        from latefuse_b200.tasks import stream_to_host

        return stream_to_host(lambda ids, mask, tenants: self.embed_tokens(ids, mask, tenants, **kw), batches, depth)
