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


def partition_rows(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Assign rows to ``world`` ranks: equal row counts (+-1, since the padded base
    forward costs the same per row), and within that the real-token load balanced
    greedily (longest rows first to the least-loaded rank with room).  Each rank's
    rows are returned in input order."""
    n = len(lengths)
    if world <= 0:
        raise ValueError("world must be positive")
    cap = [n // world + (1 if r < n % world else 0) for r in range(world)]
    parts: list[list[int]] = [[] for _ in range(world)]
    load = [0] * world
    for i in sorted(range(n), key=lambda k: -int(lengths[k])):
        r = min((k for k in range(world) if len(parts[k]) < cap[k]), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(p) for p in parts]


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

    def embed_tokens(self, input_ids: Tensor, attention_mask: Tensor, tenants: Sequence[str], **kw) -> Tensor:
        """Embed a global pre-tokenized batch (host tensors; every rank passes the same batch)."""
        lengths = attention_mask.sum(1).tolist()
        parts = partition_rows(lengths, self.world)
        mine = parts[self.rank]
        idx = torch.tensor(mine, dtype=torch.long)
        local = self.embedder.embed_tokens(input_ids[idx], attention_mask[idx], [tenants[i] for i in mine], **kw)
        rows = all_gather_rows(local, [len(p) for p in parts], self.group)
        order = torch.tensor([i for p in parts for i in p], dtype=torch.long, device=rows.device)
        out = torch.empty_like(rows)
        out[order] = rows
        return out
