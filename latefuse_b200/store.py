"""Slot-indexed adapter cache (mirror of ``src/latefuse/weights/store.py``).

Every resident adapter occupies one *slot* of a single contiguous device
buffer laid out as::

    cache[slot][module] = [ A (L, H, R) | B (L, R, H) ]      module in target_modules order

``AdapterStore.get(id).wa[m]`` / ``.wb[m]`` are contiguous views of that slot
with exactly the reference's ``LoraWeight`` shapes and layouts
(``src/latefuse/weights/store.py:22-39``), so code that fills or perturbs them
in place behaves as it does against the reference.  The kernels address a
tenant's factors as ``base + slot * slot_stride + ...``: no per-batch gather and
no re-pack after registration (the reference re-stacks the whole store,
``src/latefuse/weights/batch.py:163-170``).

On CUDA the buffer is a :class:`~latefuse_b200.arena.DeviceArena` (grows in
place).  A CPU store is supported for registration bookkeeping only; it grows by
reallocation and refreshes the views of every resident adapter.
"""

from __future__ import annotations

import heapq
from collections.abc import Callable

import torch
from torch import Tensor

from latefuse_b200.config import LoraServingConfig
from latefuse_b200.lora import FactorCache

#: Maps (layer_idx, module_name) -> (key_A, key_B) in an adapter state dict.
KeyResolverFn = Callable[[int, str], tuple[str, str]]


class LoraWeight:
    """The A and B low-rank matrices of one adapter, per target module per layer.

    Shapes (one entry per target module):
        wa[module]: (num_layers, hidden_size, lora_rank)  -- A matrix (shrink)
        wb[module]: (num_layers, lora_rank, hidden_size)  -- B matrix (expand)

    A ``LoraWeight`` returned by :meth:`AdapterStore.get` views its cache slot; one
    built directly (``LoraWeight(config)``) owns zero-initialised tensors until it
    is passed to :meth:`AdapterStore.insert`, which moves it into a slot.
    """

    def __init__(self, config: LoraServingConfig):
        H, R, L = config.hidden_size, config.lora_rank, config.num_layers
        self.wa: dict[str, Tensor] = {
            m: torch.zeros(L, H, R, dtype=config.dtype, device=config.device) for m in config.target_modules
        }
        self.wb: dict[str, Tensor] = {
            m: torch.zeros(L, R, H, dtype=config.dtype, device=config.device) for m in config.target_modules
        }

    @classmethod
    def _over(cls, wa: dict[str, Tensor], wb: dict[str, Tensor]) -> LoraWeight:
        obj = cls.__new__(cls)
        obj.wa = wa
        obj.wb = wb
        return obj

    def copy_from_tensors(self, a_by_module: dict[str, Tensor], b_by_module: dict[str, Tensor],
                          scale: float = 1.0) -> None:
        """Load from column-major tensors (as stored in adapter files).

        Args:
            a_by_module: module -> (num_layers, rank, hidden_size)
            b_by_module: module -> (num_layers, hidden_size, rank)
            scale:       alpha / rank, folded into B (same arithmetic as the
                         reference: cast to the model dtype, transpose, multiply).

        A rank below the slot's is zero-padded: A's extra columns and B's extra
        rows are zero, so ``B A x`` is unchanged (exactly) and nothing of a
        previous occupant of the slot survives.
        """
        for m, a in a_by_module.items():
            r = a.shape[1]
            if r == self.wa[m].shape[2]:
                self.wa[m].copy_(a.to(self.wa[m].device, self.wa[m].dtype).transpose(1, 2))
            else:
                self.wa[m].zero_()
                self.wa[m][:, :, :r].copy_(a.to(self.wa[m].device, self.wa[m].dtype).transpose(1, 2))
        for m, b in b_by_module.items():
            r = b.shape[2]
            if r == self.wb[m].shape[1]:
                self.wb[m].copy_(b.to(self.wb[m].device, self.wb[m].dtype).transpose(1, 2))
            else:
                self.wb[m].zero_()
                self.wb[m][:, :r, :].copy_(b.to(self.wb[m].device, self.wb[m].dtype).transpose(1, 2))
            if scale != 1.0:
                self.wb[m].mul_(scale)


class AdapterStore:
    """Resident tenant adapters in one slot-indexed device cache.

    Same interface as the reference's ``AdapterStore``
    (``src/latefuse/weights/store.py:59-207``), plus the slot accessors the
    kernels use (:meth:`slot_of`, :meth:`slots`, :meth:`factor_cache`).

    Args:
        capacity: slots to map up front (the cache grows on demand either way).
        growth:   factor by which mapped capacity grows when it runs out.
    """

    def __init__(self, config: LoraServingConfig, capacity: int | None = None, growth: float = 1.25):
        self._config = config
        M, L = len(config.target_modules), config.num_layers
        H, R = config.hidden_size, config.lora_rank
        self._M, self._L, self._H, self._R = M, L, H, R
        self._module_index = {m: i for i, m in enumerate(config.target_modules)}
        self.factor_elems = L * H * R  # elements of one (L, H, R) A block (= one B block)
        self.slot_elems = M * 2 * self.factor_elems
        self._elem = torch.empty((), dtype=config.dtype).element_size()
        self.slot_bytes = self.slot_elems * self._elem
        self._growth = max(1.01, float(growth))
        self._slot_of: dict[str, int] = {}
        self._weights: dict[str, LoraWeight] = {}
        self._free: list[int] = []
        self._next = 0
        self._arena = None
        self._buf: Tensor | None = None
        self._n_slots = 0
        self._device = torch.device(config.device)
        if self._device.type == "cuda" and self._device.index is None:
            self._device = torch.device("cuda", torch.cuda.current_device())
        if self._device.type == "cuda":
            from latefuse_b200.arena import DeviceArena

            total = torch.cuda.get_device_properties(self._device).total_memory
            self._arena = DeviceArena(self._device, reserve_bytes=max(total, self.slot_bytes * 2))
        self._ensure_slots(max(1, int(capacity or 16)))

    # -- storage -----------------------------------------------------------
    def _ensure_slots(self, n: int) -> None:
        if n <= self._n_slots:
            return
        if self._n_slots:
            n = max(n, int(self._n_slots * self._growth) + 1)
        if self._arena is not None:
            self._arena.grow(n * self.slot_bytes)
            raw = self._arena.tensor(n * self.slot_bytes)
            self._buf = raw.view(self._config.dtype).view(n, self._M, 2, self.factor_elems)
            self._n_slots = n
            return
        buf = torch.zeros(n, self._M, 2, self.factor_elems, dtype=self._config.dtype, device=self._device)
        if self._buf is not None:
            buf[: self._n_slots].copy_(self._buf)
        self._buf = buf
        self._n_slots = n
        for aid, slot in self._slot_of.items():  # CPU reallocation: refresh every view
            self._bind(self._weights[aid], slot)

    def _views(self, slot: int) -> tuple[dict[str, Tensor], dict[str, Tensor]]:
        L, H, R = self._L, self._H, self._R
        wa = {m: self._buf[slot, i, 0].view(L, H, R) for m, i in self._module_index.items()}
        wb = {m: self._buf[slot, i, 1].view(L, R, H) for m, i in self._module_index.items()}
        return wa, wb

    def _bind(self, weight: LoraWeight, slot: int) -> None:
        wa, wb = self._views(slot)
        weight.wa.clear()
        weight.wa.update(wa)
        weight.wb.clear()
        weight.wb.update(wb)

    def _claim(self, adapter_id: str) -> tuple[int, LoraWeight]:
        """Slot for ``adapter_id`` (its current one if resident) and a LoraWeight viewing it."""
        if adapter_id in self._slot_of:
            slot = self._slot_of[adapter_id]
            return slot, self._weights[adapter_id]
        if self._free:
            slot = heapq.heappop(self._free)
        else:
            slot = self._next
            self._next += 1
            self._ensure_slots(self._next)
        wa, wb = self._views(slot)
        return slot, LoraWeight._over(wa, wb)

    def _commit(self, adapter_id: str, slot: int, weight: LoraWeight) -> None:
        self._slot_of[adapter_id] = slot
        self._weights[adapter_id] = weight

    # -- registration (reference API) --------------------------------------
    def load_from_file(self, adapter_id: str, path: str, key_fn: KeyResolverFn,
                       lora_alpha: float | None = None) -> None:
        """Load a LoRA adapter from a torch ``.bin`` state dict into a slot."""
        state_dict = torch.load(path, map_location=self._device, weights_only=True)
        self.load_from_state_dict(adapter_id, state_dict, key_fn, lora_alpha=lora_alpha)

    def load_from_state_dict(self, adapter_id: str, state_dict: dict, key_fn: KeyResolverFn,
                             lora_alpha: float | None = None, pad_rank: bool = False) -> None:
        """Cache an adapter from an already-loaded state dict.

        ``alpha / rank`` is folded into B at load time, as in the reference
        (``src/latefuse/weights/store.py:104-145``).  With ``pad_rank`` an adapter
        of a lower rank ``r`` is zero-padded into the slot (mixed-rank serving:
        the delta ``(alpha / r) B A x`` is exactly that of the rank-``r`` adapter).
        """
        cfg = self._config
        a_by_module: dict[str, Tensor] = {}
        b_by_module: dict[str, Tensor] = {}
        for module in cfg.target_modules:
            a_tensors, b_tensors = [], []
            for i in range(cfg.num_layers):
                key_a, key_b = key_fn(i, module)
                for key in (key_a, key_b):
                    if key not in state_dict:
                        raise KeyError(
                            f"adapter '{adapter_id}' has no tensor '{key}'. The key layout does not "
                            f"match this key_fn; available keys start with "
                            f"{sorted(state_dict)[:3] if state_dict else '[]'}"
                        )
                a_tensors.append(state_dict[key_a])
                b_tensors.append(state_dict[key_b])
            a_by_module[module] = torch.stack(a_tensors)
            b_by_module[module] = torch.stack(b_tensors)
        ranks = {a.shape[1] for a in a_by_module.values()} | {b.shape[2] for b in b_by_module.values()}
        if len(ranks) != 1:
            raise ValueError(f"adapter '{adapter_id}' mixes ranks {sorted(ranks)} across its modules")
        rank = ranks.pop()
        if rank > cfg.lora_rank or (rank < cfg.lora_rank and not pad_rank):
            raise ValueError(
                f"adapter '{adapter_id}' has rank {rank} but this store serves rank {cfg.lora_rank}"
                + ("" if rank > cfg.lora_rank else "; pass pad_rank=True to zero-pad it into a slot")
            )
        scale = 1.0 if lora_alpha is None else lora_alpha / rank
        slot, weight = self._claim(adapter_id)
        weight.copy_from_tensors(a_by_module, b_by_module, scale=scale)
        self._commit(adapter_id, slot, weight)

    def load_synthetic(self, adapter_id: str, seed: int | None = None) -> None:
        """Random adapter for benchmarking: A ~ N(0, 0.02), B = 0.

        Draws with the global torch RNG on the store's device, module by module
        in ``target_modules`` order, into contiguous ``(L, H, R)`` blocks -- the
        same draws the reference makes (``src/latefuse/weights/store.py:147-156``).
        """
        if seed is not None:
            torch.manual_seed(seed)
        slot, weight = self._claim(adapter_id)
        for m in self._config.target_modules:
            torch.nn.init.normal_(weight.wa[m], std=0.02)
            torch.nn.init.zeros_(weight.wb[m])
        self._commit(adapter_id, slot, weight)

    def insert(self, adapter_id: str, weight: LoraWeight) -> None:
        """Make an already-populated ``LoraWeight`` resident under ``adapter_id``.

        Its tensors are copied into a slot and the object is re-pointed at the
        slot, so later in-place edits through it reach the cache.
        """
        slot, view = self._claim(adapter_id)
        for m in self._config.target_modules:
            view.wa[m].copy_(weight.wa[m])
            view.wb[m].copy_(weight.wb[m])
        if view is not weight:
            self._bind(weight, slot)
        self._commit(adapter_id, slot, weight)

    # -- lookup --------------------------------------------------------------
    @property
    def config(self) -> LoraServingConfig:
        return self._config

    def get(self, adapter_id: str) -> LoraWeight:
        """Retrieve a resident adapter by ID (views of its slot)."""
        if adapter_id not in self._slot_of:
            raise KeyError(f"Adapter '{adapter_id}' not found. Call load_from_file() or load_synthetic() first.")
        return self._weights[adapter_id]

    def evict(self, adapter_id: str) -> None:
        """Release a resident adapter's slot for reuse (its memory is not cleared)."""
        if adapter_id not in self._slot_of:
            raise KeyError(f"Adapter '{adapter_id}' is not resident.")
        slot = self._slot_of.pop(adapter_id)
        del self._weights[adapter_id]
        heapq.heappush(self._free, slot)

    def adapter_ids(self) -> list[str]:
        """All resident adapter IDs in insertion order."""
        return list(self._slot_of.keys())

    def __len__(self) -> int:
        return len(self._slot_of)

    def __contains__(self, adapter_id: object) -> bool:
        return adapter_id in self._slot_of

    def memory_bytes(self) -> int:
        """Bytes of adapter data held by resident adapters (slots in use)."""
        return len(self._slot_of) * self.slot_bytes

    def memory_gb(self) -> float:
        return self.memory_bytes() / 1e9

    # -- slot access (kernels) ---------------------------------------------
    def slot_of(self, adapter_id: str) -> int:
        try:
            return self._slot_of[adapter_id]
        except KeyError:
            raise KeyError(
                f"Adapter '{adapter_id}' not found. Call load_from_file() or load_synthetic() first."
            ) from None

    def slots(self, adapter_ids) -> list[int]:
        return [self.slot_of(a) for a in adapter_ids]

    @property
    def n_slots(self) -> int:
        """Mapped slots (valid slot ids are ``[0, n_slots)``)."""
        return self._n_slots

    @property
    def cache(self) -> Tensor:
        """The whole cache, ``(n_slots, n_modules, 2, L*H*R)``."""
        return self._buf

    def module_index(self, module: str) -> int:
        return self._module_index[module]

    def factor_cache(self, layer: int) -> FactorCache:
        """Kernel view of layer ``layer``'s factors across all slots and modules."""
        L, H, R = self._L, self._H, self._R
        return FactorCache(
            a=self._buf, b=self._buf,
            a_offset=layer * H * R, b_offset=self.factor_elems + layer * R * H,
            a_slot_stride=self.slot_elems, b_slot_stride=self.slot_elems,
            a_module_stride=2 * self.factor_elems, b_module_stride=2 * self.factor_elems,
            n_slots=self._n_slots, hidden=H, rank=R,
        )

    def fill_random_(self, n: int, std: float = 0.02, generator: torch.Generator | None = None,
                     prefix: str = "adapter_", ids: list[str] | None = None) -> list[str]:
        """Register ``n`` adapters ``{prefix}{i}`` (or the given ``ids``) with A and B both
        ~ N(0, std), drawn in one pass over the cache (a fast path for large synthetic
        populations)."""
        if ids is None:
            ids = [f"{prefix}{i}" for i in range(n)]
        elif len(ids) != n or len(set(ids)) != n:
            raise ValueError(f"ids must be {n} distinct adapter ids")
        # every id is checked before any slot is drawn or committed, so a refused
        # call leaves the store exactly as it was
        clash = next((aid for aid in ids if aid in self._slot_of), None)
        if clash is not None:
            raise ValueError(f"adapter '{clash}' is already resident")
        start = self._next
        self._ensure_slots(start + n)
        self._buf[start : start + n].normal_(0.0, std, generator=generator)
        for i, aid in enumerate(ids):
            slot = start + i
            wa, wb = self._views(slot)
            self._commit(aid, slot, LoraWeight._over(wa, wb))
        self._next = start + n
        return ids
