"""Registration of PEFT-trained adapters into the slot cache.

A registration is a file read followed by one copy into a cache slot:

1. ``adapter_config.json`` (rank ``r``, ``lora_alpha``, ``target_modules``) is
   checked against the serving config before anything is read or written.
2. Every ``lora_A`` / ``lora_B`` tensor of the weights file is read on the host
   once (a ``.safetensors`` file key by key, a ``.bin`` file memory-mapped) and
   written straight into a *slot image* in pinned host memory: the slot's own
   device layout ``[module][A (L, H, R) | B (L, R, H)]``, transposed, cast to the
   model dtype, ``alpha / r`` folded into B, and a rank below the store's
   zero-padded.
3. One host-to-device copy (``lf_cache_write_slot``) moves the whole image into
   the slot on the current stream.  Two images alternate, each guarded by an
   event, so the host reads the next file while the previous copy runs.

The file format is PEFT's, as the reference reads it
(``src/latefuse/loaders.py:35-190``): keys
``base_model.model.encoder.layer.{i}.{projection}.lora_{A,B}[.{name}].weight``
with A ``(r, H)`` and B ``(H, r)``.  The arithmetic of the fold is the
reference's (``src/latefuse/weights/store.py:36-56``: cast to the model dtype,
transpose, multiply by ``alpha / r`` in the model dtype), so a slot holds the
same bits the reference's ``LoraWeight`` would.  The reference stages nothing
in its library path; its churn benchmark's pinned arm
(``src/latefuse/benchmark/churn.py:175-286``) copies module by module through
pinned buffers, which is what this path turns into one copy per adapter.
"""

from __future__ import annotations

import json
import os
import warnings
from dataclasses import dataclass

import torch

from latefuse_b200.engine import _TARGET_SUFFIXES
from latefuse_b200.store import AdapterStore

#: weight files of a PEFT adapter directory, the first one present is read
WEIGHT_FILES = ("adapter_model.safetensors", "adapter_model.bin")


def peft_key_fn(model_type: str, adapter_name: str = "default"):
    """``(layer, module) -> (A key, B key)`` in PEFT's state-dict naming for ``model_type``.

    ``adapter_name`` appears in the keys only when PEFT saved several adapters of
    one model; the default single-adapter save omits it.
    """
    projection = _TARGET_SUFFIXES.get(model_type, _TARGET_SUFFIXES["default"])
    tag = "" if adapter_name in (None, "", "default") else "." + adapter_name

    def keys(layer: int, module: str) -> tuple[str, str]:
        if module not in projection:
            raise ValueError(f"target module '{module}' has no mapping for model_type '{model_type}' "
                             f"(known: {sorted(projection)})")
        prefix = f"base_model.model.encoder.layer.{layer}.{projection[module]}"
        return f"{prefix}.lora_A{tag}.weight", f"{prefix}.lora_B{tag}.weight"

    return keys


@dataclass(frozen=True)
class PeftAdapterConfig:
    """The fields of ``adapter_config.json`` that decide whether an adapter can be served."""

    rank: int | None = None
    alpha: float | None = None
    targets: tuple[str, ...] | None = None

    @classmethod
    def read(cls, directory: str) -> PeftAdapterConfig | None:
        path = os.path.join(directory, "adapter_config.json")
        if not os.path.exists(path):
            return None
        with open(path) as fh:
            raw = json.load(fh)
        targets = raw.get("target_modules")
        return cls(rank=raw.get("r"), alpha=raw.get("lora_alpha"),
                   targets=None if targets is None else tuple(str(t) for t in targets))

    def mismatches(self, rank: int, targets, pad_rank: bool) -> list[str]:
        """Why this adapter cannot be served by a pipeline of ``rank`` on ``targets``.

        Target names are compared without the ``_proj`` suffix some architectures
        use in their checkpoints (``query_proj`` is the logical ``query``).
        """
        out = []
        if self.rank is not None and self.rank != rank and not (pad_rank and self.rank < rank):
            hint = "; pass pad_rank=True to zero-pad it into this pipeline's slots" if self.rank < rank else ""
            out.append(f"it was trained at rank {self.rank} and this pipeline serves rank {rank} "
                       f"(one pipeline serves one rank{hint})")
        if self.targets is not None:
            have = sorted({t.removesuffix("_proj") for t in self.targets})
            want = sorted({str(t).removesuffix("_proj") for t in targets})
            if have != want:
                out.append(f"it adapts {have} and this pipeline adapts {want}, so its deltas would land on the "
                           "wrong projections")
        return out


def _weights_file(path: str) -> str:
    if not os.path.isdir(path):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        return path
    for name in WEIGHT_FILES:
        if os.path.exists(os.path.join(path, name)):
            return os.path.join(path, name)
    raise FileNotFoundError(f"{path} holds none of {list(WEIGHT_FILES)}; expected a PEFT adapter directory")


class _TensorSource:
    """Host tensors of a weights file by key, read lazily (safetensors) or memory-mapped (.bin)."""

    def __init__(self, path: str):
        self._st = None
        if path.endswith(".safetensors"):
            from safetensors import safe_open

            self._st = safe_open(path, framework="pt", device="cpu")
            self._keys = set(self._st.keys())
        else:
            try:
                self._sd = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
            except RuntimeError:  # an old (non-zip) serialisation cannot be memory-mapped
                self._sd = torch.load(path, map_location="cpu", weights_only=True)
            self._keys = set(self._sd)

    def __contains__(self, key: str) -> bool:
        return key in self._keys

    def __getitem__(self, key: str) -> torch.Tensor:
        return self._st.get_tensor(key) if self._st is not None else self._sd[key]

    def sample_keys(self) -> list[str]:
        return sorted(self._keys)[:3]


class AdapterRegistrar:
    """Registers adapter files into one :class:`AdapterStore` through pinned slot images.

    One registrar per store; :func:`load_peft_adapter` keeps one on the store.
    A registration returns once its copy is queued on the current stream: kernels
    queued after it on that stream see the adapter.
    """

    def __init__(self, store: AdapterStore, images: int = 2):
        self.store = store
        cfg = store.config
        self._cuda = store.cache.device.type == "cuda"
        shape = (len(cfg.target_modules), 2, store.factor_elems)
        self._images = [torch.empty(shape, dtype=cfg.dtype, pin_memory=self._cuda) for _ in range(max(1, images))]
        self._done = [None] * len(self._images)
        self._turn = 0

    def _image(self) -> torch.Tensor:
        i = self._turn
        self._turn = (i + 1) % len(self._images)
        if self._done[i] is not None:
            self._done[i].synchronize()  # the copy that last read this image has finished
        return i, self._images[i]

    def stage(self, image: torch.Tensor, source, key_fn, rank: int, scale: float, adapter_id: str) -> None:
        """Fill a slot image from ``source[key]`` tensors (A ``(r, H)``, B ``(H, r)``)."""
        cfg = self.store.config
        L, H, R = cfg.num_layers, cfg.hidden_size, cfg.lora_rank
        for mi, module in enumerate(cfg.target_modules):
            a_img = image[mi, 0].view(L, H, R)
            b_img = image[mi, 1].view(L, R, H)
            if rank < R:  # nothing of a previous occupant may survive in the padding
                a_img[:, :, rank:].zero_()
                b_img[:, rank:, :].zero_()
            for layer in range(L):
                key_a, key_b = key_fn(layer, module)
                for key in (key_a, key_b):
                    if key not in source:
                        raise KeyError(f"adapter '{adapter_id}' has no tensor '{key}'. The key layout does not "
                                       f"match this key_fn; available keys start with {source.sample_keys()}")
                a, b = source[key_a], source[key_b]
                if tuple(a.shape) != (rank, H) or tuple(b.shape) != (H, rank):
                    raise ValueError(f"adapter '{adapter_id}': {key_a} is {tuple(a.shape)} and {key_b} is "
                                     f"{tuple(b.shape)}; expected ({rank}, {H}) and ({H}, {rank}) at rank {rank}")
                a_img[layer, :, :rank].copy_(a.t())
                b_img[layer, :rank, :].copy_(b.t())
            if scale != 1.0:
                b_img[:, :rank, :].mul_(scale)  # in the model dtype, after the cast, as the reference folds it

    def commit(self, adapter_id: str, index: int, image: torch.Tensor) -> None:
        """Copy a staged image into ``adapter_id``'s slot and make it resident."""
        store = self.store
        slot, weight = store._claim(adapter_id)
        if self._cuda:
            from latefuse_b200 import _native as nat

            stream = torch.cuda.current_stream(store.cache.device)
            nat.check(nat.lib().lf_cache_write_slot(stream.cuda_stream, store.cache.data_ptr(), store.slot_bytes,
                                                    slot, store.n_slots, 0, image.data_ptr(), store.slot_bytes),
                      "lf_cache_write_slot")
            ev = torch.cuda.Event()
            ev.record(stream)
            self._done[index] = ev
        else:
            store.cache[slot].copy_(image)
        store._commit(adapter_id, slot, weight)

    def register(self, adapter_id: str, path: str, *, adapter_name: str = "default",
                 lora_alpha: float | None = None, strict: bool = True, pad_rank: bool = False) -> None:
        """Check, stage and copy one PEFT adapter (directory or weights file) into a slot."""
        cfg = self.store.config
        directory = path if os.path.isdir(path) else (os.path.dirname(path) or ".")
        meta = PeftAdapterConfig.read(directory)
        if meta is not None:
            problems = meta.mismatches(cfg.lora_rank, cfg.target_modules, pad_rank)
            if problems:
                msg = f"adapter '{adapter_id}' does not fit this pipeline: " + "; ".join(problems) + "."
                if strict:
                    raise ValueError(msg + " Pass strict=False to load anyway.")
                warnings.warn(msg, stacklevel=3)
        alpha = lora_alpha if lora_alpha is not None else (meta.alpha if meta is not None else None)
        source = _TensorSource(_weights_file(path))
        key_fn = peft_key_fn(cfg.hf_config.model_type, adapter_name)
        first = key_fn(0, cfg.target_modules[0])[0]
        rank = source[first].shape[0] if first in source else cfg.lora_rank  # stage() reports a missing key
        if rank > cfg.lora_rank or (rank < cfg.lora_rank and not (pad_rank or not strict)):
            raise ValueError(f"adapter '{adapter_id}' has rank {rank} but this store serves rank {cfg.lora_rank}"
                             + ("" if rank > cfg.lora_rank else "; pass pad_rank=True to zero-pad it into a slot"))
        scale = 1.0 if alpha is None else alpha / rank
        index, image = self._image()
        self.stage(image, source, key_fn, rank, scale, adapter_id)
        self.commit(adapter_id, index, image)


def registrar_for(store: AdapterStore) -> AdapterRegistrar:
    """The store's registrar (created on first use; its pinned images live as long as the store)."""
    reg = getattr(store, "_registrar", None)
    if reg is None:
        reg = AdapterRegistrar(store)
        store._registrar = reg
    return reg


def load_peft_adapter(store: AdapterStore, adapter_id: str, path: str, *, adapter_name: str = "default",
                      lora_alpha: float | None = None, strict: bool = True, pad_rank: bool = False) -> None:
    """Make the PEFT adapter at ``path`` (directory or weights file) resident in ``store``.

    The adapter's ``adapter_config.json``, when present, must match the store's
    rank and target modules (``strict``; otherwise a warning), its ``lora_alpha``
    is folded into B unless ``lora_alpha`` overrides it, and with ``pad_rank`` a
    lower-rank adapter is zero-padded into its slot (the delta is unchanged).

    Raises:
        ValueError:        the adapter does not fit the pipeline (rank, targets, shapes).
        FileNotFoundError: no weights file at ``path``.
        KeyError:          the weights lack a layer's key.
    """
    registrar_for(store).register(adapter_id, path, adapter_name=adapter_name, lora_alpha=lora_alpha,
                                  strict=strict, pad_rank=pad_rank)
