"""Mixed-rank serving from native-rank buckets.

The reference measures two ways to serve a fleet whose adapters have different ranks
(``benchmarks/profiling/mixed_rank_bench.py:320-431``): every adapter zero-padded to
the largest rank in one store ("padded": here ``AdapterStore.load_from_state_dict(...,
pad_rank=True)``), or each adapter kept at its own rank in a bucket of that rank and
padded per batch (``PadToMaxAssembler``: per rank present, one gather of the bucket's
rows, zero-extended to r_max and scattered to their batch positions).

:class:`RankBucketStore` is the second form.  Each rank's adapters live in their own
:class:`~latefuse_b200.store.AdapterStore` (slot cache at that rank), so a rank-4
adapter in an r_max-32 fleet takes an eighth of a padded slot.  Per batch,
:meth:`RankBucketStore.batch_store` gathers the batch's distinct adapters into one
staging cache at r_max -- per rank present, one ``index_select`` from that bucket's
cache and one scatter into the staging rows (the padded columns zeroed) -- and returns
it as a store the engines serve from unchanged (slot ids are positions in the staging
cache).  The staging cache is reused from batch to batch; every step on it is ordered
on the current stream after the previous batch's kernels, and each batch re-zeroes the
rows it uses, so no earlier occupant's columns leak into a lower-rank adapter.
"""

from __future__ import annotations

import dataclasses
from collections.abc import Iterable, Sequence

import torch

from latefuse_b200.config import LoraServingConfig
from latefuse_b200.store import AdapterStore, KeyResolverFn, LoraWeight


class _BatchStage(AdapterStore):
    """The r_max staging cache of one batch: adapter ``batch_ids[u]`` in slot ``u``."""

    def _set_batch(self, batch_ids: Sequence[str]) -> None:
        self._slot_of = {a: u for u, a in enumerate(batch_ids)}
        self._weights = {}
        self._next = len(batch_ids)

    def get(self, adapter_id: str) -> LoraWeight:
        w = self._weights.get(adapter_id)
        if w is None:
            w = LoraWeight._over(*self._views(self.slot_of(adapter_id)))
            self._weights[adapter_id] = w
        return w

    def load_from_state_dict(self, *args, **kwargs):
        raise TypeError("a batch's staging cache is filled by RankBucketStore.batch_store")

    load_synthetic = load_from_state_dict
    insert = load_from_state_dict
    fill_random_ = load_from_state_dict


class RankBucketStore:
    """Adapters of ranks up to ``config.lora_rank``, each stored at its own rank.

    Registration mirrors :class:`~latefuse_b200.store.AdapterStore` (the rank is read
    from the adapter); serving goes through :meth:`batch_store`, which the task
    pipelines call for every batch.
    """

    def __init__(self, config: LoraServingConfig, capacity: int | None = None):
        self._config = config
        self._capacity = capacity
        self._buckets: dict[int, AdapterStore] = {}
        self._rank_of: dict[str, int] = {}
        self._stage: _BatchStage | None = None

    # -- buckets --------------------------------------------------------------
    def _bucket(self, rank: int) -> AdapterStore:
        if rank < 1 or rank > self._config.lora_rank:
            raise ValueError(f"rank {rank} is outside 1..{self._config.lora_rank}, the ranks this store serves")
        b = self._buckets.get(rank)
        if b is None:
            b = AdapterStore(dataclasses.replace(self._config, lora_rank=rank), capacity=self._capacity)
            self._buckets[rank] = b
        return b

    def _settle(self, adapter_id: str, rank: int) -> None:
        """After ``adapter_id`` was made resident in the rank-``rank`` bucket: leave any
        other bucket it was in (a failed registration changes nothing)."""
        old = self._rank_of.get(adapter_id)
        if old is not None and old != rank:
            self._buckets[old].evict(adapter_id)
        self._rank_of[adapter_id] = rank

    @property
    def config(self) -> LoraServingConfig:
        return self._config

    def ranks(self) -> list[int]:
        """Ranks with at least one resident adapter."""
        return sorted({r for r in self._rank_of.values()})

    def rank_of(self, adapter_id: str) -> int:
        try:
            return self._rank_of[adapter_id]
        except KeyError:
            raise KeyError(f"Adapter '{adapter_id}' not found. Call load_from_file() or load_synthetic() first.") \
                from None

    # -- registration -----------------------------------------------------------
    def load_from_state_dict(self, adapter_id: str, state_dict: dict, key_fn: KeyResolverFn,
                             lora_alpha: float | None = None) -> None:
        """Cache an adapter at its own rank (read from its first module's A)."""
        key_a, _ = key_fn(0, self._config.target_modules[0])
        if key_a not in state_dict:
            raise KeyError(f"adapter '{adapter_id}' has no tensor '{key_a}'")
        rank = int(state_dict[key_a].shape[0])
        self._bucket(rank).load_from_state_dict(adapter_id, state_dict, key_fn, lora_alpha)
        self._settle(adapter_id, rank)

    def load_peft(self, adapter_id: str, path: str, *, adapter_name: str = "default",
                  lora_alpha: float | None = None, strict: bool = True) -> None:
        """A PEFT adapter (directory or weights file) into the bucket of its rank, through
        that bucket's pinned-staging registrar (``load_peft_adapter`` routes here)."""
        from latefuse_b200.loaders import peft_rank, registrar_for

        rank = peft_rank(path, self._config, adapter_name)
        registrar_for(self._bucket(rank)).register(adapter_id, path, adapter_name=adapter_name,
                                                   lora_alpha=lora_alpha, strict=strict)
        self._settle(adapter_id, rank)

    def load_from_file(self, adapter_id: str, path: str, key_fn: KeyResolverFn,
                       lora_alpha: float | None = None) -> None:
        from safetensors.torch import load_file

        self.load_from_state_dict(adapter_id, load_file(path), key_fn, lora_alpha)

    def load_synthetic(self, adapter_id: str, seed: int | None = None, rank: int | None = None) -> None:
        """Random adapter of ``rank`` (default the largest): A ~ N(0, 0.02), B = 0."""
        rank = rank or self._config.lora_rank
        self._bucket(rank).load_synthetic(adapter_id, seed=seed)
        self._settle(adapter_id, rank)

    def fill_random_(self, ranks: Iterable[int], std: float = 0.02, generator: torch.Generator | None = None,
                     prefix: str = "adapter_") -> list[str]:
        """Register ``{prefix}{i}`` with rank ``ranks[i]``, A and B ~ N(0, std): each
        rank's adapters drawn in one pass over that bucket."""
        ranks = list(ranks)
        ids = [f"{prefix}{i}" for i in range(len(ranks))]
        clash = [a for a in ids if a in self._rank_of]
        if clash:
            raise ValueError(f"already resident: {clash[:5]}")
        for r in sorted(set(ranks)):
            mine = [ids[i] for i, ri in enumerate(ranks) if ri == r]
            self._bucket(r).fill_random_(len(mine), std=std, generator=generator, ids=mine)
            for aid in mine:
                self._rank_of[aid] = r
        return ids

    def get(self, adapter_id: str) -> LoraWeight:
        """The adapter at its own rank (views of its bucket slot)."""
        return self._buckets[self.rank_of(adapter_id)].get(adapter_id)

    def evict(self, adapter_id: str) -> None:
        if adapter_id not in self._rank_of:
            raise KeyError(f"Adapter '{adapter_id}' is not resident.")
        self._buckets[self._rank_of.pop(adapter_id)].evict(adapter_id)

    def adapter_ids(self) -> list[str]:
        return list(self._rank_of)

    def __len__(self) -> int:
        return len(self._rank_of)

    def __contains__(self, adapter_id: object) -> bool:
        return adapter_id in self._rank_of

    def memory_bytes(self) -> int:
        """Bytes of adapter data held at native ranks (the staging cache not counted)."""
        return sum(b.memory_bytes() for b in self._buckets.values())

    def memory_gb(self) -> float:
        return self.memory_bytes() / 1e9

    def slots(self, adapter_ids) -> list[int]:
        raise TypeError("RankBucketStore serves through batch_store(adapter_ids); its buckets' slots are per rank")

    # -- serving ------------------------------------------------------------------
    def batch_store(self, adapter_ids: Sequence[str]) -> AdapterStore:
        """A store holding this batch's distinct adapters zero-padded to r_max in slots
        0..U-1 (grouped by rank; ``slots(ids)`` gives each one's), as the reference's
        ``PadToMaxAssembler`` pads them: per rank present, one gather from its bucket
        and a strided copy into the padded rows, the columns past the rank zeroed."""
        distinct = list(dict.fromkeys(adapter_ids))
        ranks = {a: self.rank_of(a) for a in distinct}  # KeyError naming an unknown tenant
        # staging slots grouped by rank, so each rank's adapters land in one contiguous
        # run of slots: one gather from the bucket, one strided copy and one zero fill
        batch_ids = sorted(distinct, key=lambda a: ranks[a])
        U = len(batch_ids)
        if self._stage is None:
            self._stage = _BatchStage(self._config, capacity=max(U, 16))
        stage = self._stage
        stage._ensure_slots(max(U, 1))
        stage._set_batch(batch_ids)
        if U == 0:
            return stage
        cfg = self._config
        M, L, H, R = len(cfg.target_modules), cfg.num_layers, cfg.hidden_size, cfg.lora_rank
        buf = stage.cache  # (n_slots, M, 2, L*H*R)
        dev = buf.device
        s0 = 0
        while s0 < U:
            r = ranks[batch_ids[s0]]
            s1 = s0
            while s1 < U and ranks[batch_ids[s1]] == r:
                s1 += 1
            bucket = self._buckets[r]
            src_slots = torch.tensor(bucket.slots(batch_ids[s0:s1]), dtype=torch.long, device=dev)
            if r == R:
                torch.index_select(bucket.cache, 0, src_slots, out=buf[s0:s1])
            else:
                n = s1 - s0
                src = bucket.cache.index_select(0, src_slots)  # (n, M, 2, L*H*r)
                dst_a = buf[s0:s1, :, 0].view(n, M, L, H, R)
                dst_b = buf[s0:s1, :, 1].view(n, M, L, R, H)
                dst_a[..., :r].copy_(src[:, :, 0].view(n, M, L, H, r))
                dst_a[..., r:].zero_()  # the columns past the rank (and any previous occupant's)
                dst_b[:, :, :, :r].copy_(src[:, :, 1].view(n, M, L, r, H))
                dst_b[:, :, :, r:].zero_()
            s0 = s1
        return stage


def store_for_batch(store, adapter_ids: Sequence[str]):
    """The store a batch is served from: ``store`` itself, or for a
    :class:`RankBucketStore` its staging cache for these adapters."""
    return store.batch_store(adapter_ids) if isinstance(store, RankBucketStore) else store


__all__ = ["RankBucketStore", "store_for_batch"]
