"""Batch assembly over the slot cache (mirror of ``src/latefuse/weights/batch.py``).

The reference assembles per-row adapter factors either with a host loop over
samples x layers x modules (``BatchAssembler``, ``:44-71``) or by re-packing the
store and gathering with ``index_select`` (``IndexSelectBatchAssembler``,
``:127-220``).  Here the factors never move: assembling a batch means mapping
tenant ids to slot ids and building a :class:`~latefuse_b200.lora.SegmentTable`
(:class:`BatchLora`), which the kernels use to read each row's factors in
place.  The reference's materialising methods are kept, bit-exact, for callers
that use them directly.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from latefuse_b200 import _native as nat
from latefuse_b200.config import LoraServingConfig
from latefuse_b200.lora import SegmentTable


class LayerwiseBatchedWeights:
    """LoRA weights for all samples in a batch, for one transformer layer.

    Each list contains one tensor per sample (``(1, H, R)`` / ``(1, R, H)``), or a
    single ``(B, H, R)`` / ``(B, R, H)`` tensor.
    """

    def __init__(self):
        self.a: dict[str, list[Tensor]] = {}
        self.b: dict[str, list[Tensor]] = {}


class BatchedLRWeights:
    """Logistic regression weights for all samples in a batch, zero-padded to max_labels."""

    coef: Tensor       # (B, max_labels, H)
    intercept: Tensor  # (B, max_labels)
    num_labels: list[int]


class BatchLora:
    """The adapter side of one mixed-tenant batch: the store's slot cache plus the
    rows' segment table.  This is what the engines consume on the serving path."""

    def __init__(self, store, segments: SegmentTable):
        self.store = store
        self.segments = segments

    @property
    def slots(self) -> list[int]:
        return self.segments.slots


class _SlotAssembler:
    def __init__(self, store, config: LoraServingConfig):
        self._store = store
        self._config = config

    def batch_lora(self, adapter_ids: list[str], seq_len: int | None = None,
                   lengths: list[int] | None = None) -> BatchLora:
        """Map one batch's tenant ids to slots (``KeyError`` for unknown ids).

        ``lengths`` (host ints) restricts each row's segment to its first
        ``lengths[i]`` tokens (right-padded rows), skipping padding.
        """
        S = seq_len if seq_len is not None else self._config.max_seq_len
        slots = self._store.slots(adapter_ids)
        segs = SegmentTable.for_padded(slots, S, self._store._device, lengths=lengths)
        return BatchLora(self._store, segs)


class BatchAssembler(_SlotAssembler):
    """Reference-compatible assembler (the ``"cpu"`` assembler name).

    :meth:`assemble_lora` returns per-layer lists of per-sample views, as the
    reference does; the serving path uses :meth:`batch_lora` instead.
    """

    def assemble_lora(self, adapter_ids: list[str]) -> list[LayerwiseBatchedWeights]:
        cfg = self._config
        lora_weights = [LayerwiseBatchedWeights() for _ in range(cfg.num_layers)]
        for module in cfg.target_modules:
            for layer_idx in range(cfg.num_layers):
                lora_weights[layer_idx].a[module] = []
                lora_weights[layer_idx].b[module] = []
        for adapter_id in adapter_ids:
            weight = self._store.get(adapter_id)
            for layer_idx in range(cfg.num_layers):
                for module in cfg.target_modules:
                    lora_weights[layer_idx].a[module].append(weight.wa[module][layer_idx].unsqueeze(0))
                    lora_weights[layer_idx].b[module].append(weight.wb[module][layer_idx].unsqueeze(0))
        return lora_weights

    def assemble_lr(self, lr_coefs: list[Tensor], lr_intercepts: list[Tensor]) -> BatchedLRWeights:
        """Stack per-sample LR heads ``(1, n, H)`` / ``(1, n)`` zero-padded to the widest."""
        num_labels = [c.shape[1] for c in lr_coefs]
        max_labels = max(num_labels)
        lr_weights = BatchedLRWeights()
        lr_weights.coef = torch.cat([F.pad(c, (0, 0, 0, max_labels - c.shape[1])) for c in lr_coefs], dim=0)
        lr_weights.intercept = torch.cat([F.pad(ic, (0, max_labels - ic.shape[1])) for ic in lr_intercepts], dim=0)
        lr_weights.num_labels = num_labels
        return lr_weights

    def assemble(self, adapter_ids, lr_coefs, lr_intercepts):
        return self.assemble_lora(adapter_ids), self.assemble_lr(lr_coefs, lr_intercepts)


class IndexSelectBatchAssembler(_SlotAssembler):
    """Device-resident assembler (the ``"index_select"`` assembler name).

    ``wa[m]`` / ``wb[m]`` are ``(n_slots, L, H, R)`` / ``(n_slots, L, R, H)`` views of
    the slot cache (nothing is packed or copied at construction) and
    :meth:`batch_index` returns slot ids, so ``wa[m][batch_index(ids)]`` is each
    row's adapter, as with the reference's packed tensors.  :meth:`assemble_lora`
    materialises the per-row factors with the native gather kernel, bit-exact.
    """

    def __init__(self, store, config: LoraServingConfig):
        super().__init__(store, config)
        L, H, R = config.num_layers, config.hidden_size, config.lora_rank
        cache = store.cache
        self.wa = {m: cache[:, store.module_index(m), 0].view(-1, L, H, R) for m in config.target_modules}
        self.wb = {m: cache[:, store.module_index(m), 1].view(-1, L, R, H) for m in config.target_modules}

    def batch_index(self, adapter_ids: list[str]) -> Tensor:
        """Slot ids of ``adapter_ids`` as a ``(B,)`` int64 tensor on the store device."""
        return torch.tensor([self._store.slot_of(a) for a in adapter_ids], dtype=torch.long,
                            device=self._config.device)

    def assemble_lora(self, adapter_ids: list[str]) -> dict[str, tuple[Tensor, Tensor]]:
        """module -> (A ``(B, L, H, R)``, B ``(B, L, R, H)``) gathered from the cache."""
        store = self._store
        slots = store.slots(adapter_ids)
        out = {}
        for m in self._config.target_modules:
            a = self.wa[m]
            b = self.wb[m]
            if a.device.type != "cuda":
                idx = torch.tensor(slots, dtype=torch.long, device=a.device)
                out[m] = (a.index_select(0, idx), b.index_select(0, idx))
                continue
            out[m] = (gather_slots(store.cache, slots, store.module_index(m), 0, a.shape[1:]),
                      gather_slots(store.cache, slots, store.module_index(m), 1, b.shape[1:]))
        return out

    def to_layerwise(self, adapter_ids: list[str]) -> list[LayerwiseBatchedWeights]:
        batched = self.assemble_lora(adapter_ids)
        layers = [LayerwiseBatchedWeights() for _ in range(self._config.num_layers)]
        for m, (a, b) in batched.items():
            for layer_idx in range(self._config.num_layers):
                layers[layer_idx].a[m] = [a[:, layer_idx]]
                layers[layer_idx].b[m] = [b[:, layer_idx]]
        return layers


def gather_slots(cache: Tensor, slots: list[int], module: int, which: int, shape) -> Tensor:
    """Copy ``cache[slot, module, which]`` for each slot into a new ``(len(slots), *shape)``
    tensor with the native gather kernel (a bit-exact copy)."""
    dev = nat.require_cuda(cache)
    n_slots = cache.shape[0]
    slot_stride = cache.stride(0)
    offset = module * cache.stride(1) + which * cache.stride(2)
    n_elems = cache.shape[3]
    out = torch.empty(len(slots), n_elems, dtype=cache.dtype, device=dev)
    if not slots:
        return out.view(0, *shape)
    idx = torch.tensor(slots, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
    rc = nat.lib().lf_cache_gather(nat.stream_ptr(dev), cache.data_ptr(), slot_stride, offset, n_elems,
                                   cache.element_size(), n_slots, idx.data_ptr(), len(slots),
                                   out.data_ptr(), None)
    nat.check(rc, "lf_cache_gather")
    return out.view(len(slots), *shape)
