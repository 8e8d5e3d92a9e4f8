"""Registration of PEFT-trained adapters into the slot cache.

A registration is a file read followed by one copy into a cache slot:

1. ``adapter_config.json`` (rank ``r``, ``lora_alpha``, ``target_modules``) is
   checked against the serving config before anything is read or written.
2. A ``.safetensors`` file is read whole, by one ``readinto``, into a reused
   pinned buffer; for a CUDA store its bytes go to the device in one copy, and
   the device casts each module's ``lora_A`` / ``lora_B`` tensors to the model
   dtype, transposes them into the slot's layout
   ``[module][A (L, H, R) | B (L, R, H)]``, folds ``alpha / r`` into B and
   zero-pads a rank below the store's, writing straight into the slot.
3. Otherwise (a ``.bin`` file, a CPU store) the same fold fills a *slot image*
   in pinned host memory and one host-to-device copy (``lf_cache_write_slot``)
   moves it into the slot.  Two images alternate, each guarded by an event, so
   the host reads the next file while the previous copy runs.

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


_SAFETENSORS_DTYPES = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "F64": torch.float64}


class _TensorSource:
    """Host tensors of a weights file by key.

    A ``.safetensors`` file (an 8-byte little-endian header length, a JSON header
    ``{key: {dtype, shape, data_offsets}}``, then the raw data) is read whole with
    one ``readinto`` into ``buffer``, a byte tensor the caller reuses from file to
    file (pinned, for a CUDA store), and every tensor is a view of it: mapping the
    file instead costs a page fault per 4 KB on every registration, several times
    the read.  A ``.bin`` file goes through ``torch.load``.
    """

    def __init__(self, path: str, buffer: torch.Tensor | None = None, pin: bool = False):
        self._st: dict | None = None
        self.buffer = buffer
        self.size = 0
        if path.endswith(".safetensors"):
            size = os.path.getsize(path)
            if self.buffer is None or self.buffer.numel() < size:
                self.buffer = torch.empty(max(size, 1 << 20), dtype=torch.uint8, pin_memory=pin)
            view = memoryview(self.buffer.numpy())[:size]
            with open(path, "rb", buffering=0) as fh:
                got = fh.readinto(view)
            if got != size:
                raise OSError(f"{path}: read {got} of {size} bytes")
            n = int.from_bytes(bytes(view[:8]), "little")
            header = json.loads(bytes(view[8 : 8 + n]))
            header.pop("__metadata__", None)
            self._st = header
            self._base = 8 + n
            self._keys = set(header)
            self.size = size
        else:
            try:
                self._sd = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
            except RuntimeError:  # an old (non-zip) serialisation cannot be memory-mapped
                self._sd = torch.load(path, map_location="cpu", weights_only=True)
            self._keys = set(self._sd)

    @property
    def raw(self) -> bool:
        """Whether every tensor is a view of :attr:`buffer` (a safetensors file)."""
        return self._st is not None

    def __contains__(self, key: str) -> bool:
        return key in self._keys

    def locate(self, key: str) -> tuple[int, torch.dtype, list[int]]:
        """(byte offset in :attr:`buffer`, dtype, shape) of a raw tensor."""
        meta = self._st[key]
        dtype = _SAFETENSORS_DTYPES.get(meta["dtype"])
        if dtype is None:
            raise ValueError(f"tensor '{key}' has dtype {meta['dtype']}; expected a floating-point LoRA factor")
        return self._base + meta["data_offsets"][0], dtype, list(meta["shape"])

    def __getitem__(self, key: str) -> torch.Tensor:
        if self._st is None:
            return self._sd[key]
        off, dtype, shape = self.locate(key)
        n = dtype.itemsize
        for d in shape:
            n *= d
        return self.buffer[off : off + n].view(dtype).view(shape)

    def shape(self, key: str) -> tuple[int, ...]:
        return tuple(self.locate(key)[2]) if self._st is not None else tuple(self._sd[key].shape)

    def sample_keys(self) -> list[str]:
        return sorted(self._keys)[:3]


class AdapterRegistrar:
    """Registers adapter files into one :class:`AdapterStore`.

    One registrar per store; :func:`load_peft_adapter` keeps one on the store.
    For a CUDA store a ``.safetensors`` file goes to the device as it is, in one
    copy from a pinned buffer, and the device casts, transposes and scales each
    module's factors straight into the slot; other files (``.bin``, or tensors
    whose offsets do not suit a device view) are staged on the host into a pinned
    image of the slot and copied with ``lf_cache_write_slot``.  Either way a
    registration returns once its work is queued on the current stream: kernels
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
        self._file_buffer: torch.Tensor | None = None  # the last weights file read, reused
        self._file_done = None                          # event: the device has copied that buffer
        self._dev_raw: torch.Tensor | None = None       # the file's bytes on the device

    def _image(self) -> torch.Tensor:
        i = self._turn
        self._turn = (i + 1) % len(self._images)
        if self._done[i] is not None:
            self._done[i].synchronize()  # the copy that last read this image has finished
        return i, self._images[i]

    def _factors(self, source, key_fn, rank: int, adapter_id: str) -> list[tuple[list[str], list[str]]]:
        """Every module's A and B keys in layer order, checked for presence and shape."""
        cfg = self.store.config
        H = cfg.hidden_size
        out = []
        for module in cfg.target_modules:
            keys_a, keys_b = [], []
            for layer in range(cfg.num_layers):
                key_a, key_b = key_fn(layer, module)
                for key in (key_a, key_b):
                    if key not in source:
                        raise KeyError(f"adapter '{adapter_id}' has no tensor '{key}'. The key layout does not "
                                       f"match this key_fn; available keys start with {source.sample_keys()}")
                sa, sb = source.shape(key_a), source.shape(key_b)
                if sa != (rank, H) or sb != (H, rank):
                    raise ValueError(f"adapter '{adapter_id}': {key_a} is {sa} and {key_b} is {sb}; expected "
                                     f"({rank}, {H}) and ({H}, {rank}) at rank {rank}")
                keys_a.append(key_a)
                keys_b.append(key_b)
            out.append((keys_a, keys_b))
        return out

    @staticmethod
    def _fold(wa: torch.Tensor, wb: torch.Tensor, a_layers, b_layers, rank: int, scale: float) -> None:
        """Write one module's factors into ``wa (L, H, R)`` / ``wb (L, R, H)``: cast to the
        model dtype, transpose, ``alpha / r`` folded into B in the model dtype (the
        reference's order), padding beyond ``rank`` zeroed.  One copy per factor."""
        R = wa.shape[2]
        if rank < R:  # nothing of a previous occupant may survive in the padding
            wa[:, :, rank:].zero_()
            wb[:, rank:, :].zero_()
        dt = wa.dtype
        wa[:, :, :rank].copy_(torch.stack(a_layers).to(dt).transpose(1, 2))
        wb[:, :rank, :].copy_(torch.stack(b_layers).to(dt).transpose(1, 2))
        if scale != 1.0:
            wb[:, :rank, :].mul_(scale)

    def stage(self, image: torch.Tensor, source, plan, rank: int, scale: float) -> None:
        """Fill a host slot image from the file's tensors."""
        cfg = self.store.config
        L, H, R = cfg.num_layers, cfg.hidden_size, cfg.lora_rank
        for mi, (keys_a, keys_b) in enumerate(plan):
            self._fold(image[mi, 0].view(L, H, R), image[mi, 1].view(L, R, H), [source[k] for k in keys_a],
                       [source[k] for k in keys_b], rank, scale)

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

    def _device_ready(self, source, plan) -> bool:
        """Whether every tensor can be viewed in place on the device (element-aligned offsets)."""
        if not (self._cuda and source.raw):
            return False
        for keys_a, keys_b in plan:
            for key in keys_a + keys_b:
                off, dtype, _ = source.locate(key)
                if off % dtype.itemsize:
                    return False
        return True

    def commit_on_device(self, adapter_id: str, source, plan, rank: int, scale: float) -> None:
        """One copy of the file's bytes to the device, then the fold into the slot there."""
        store = self.store
        dev = store.cache.device
        stream = torch.cuda.current_stream(dev)
        if self._dev_raw is None or self._dev_raw.numel() < source.size:
            self._dev_raw = torch.empty(source.buffer.numel(), dtype=torch.uint8, device=dev)
        raw = self._dev_raw
        raw[: source.size].copy_(source.buffer[: source.size], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._file_done = ev  # the next read into the pinned buffer waits for this copy

        def view(key: str) -> torch.Tensor:
            off, dtype, shape = source.locate(key)
            n = dtype.itemsize
            for d in shape:
                n *= d
            return raw[off : off + n].view(dtype).view(shape)

        slot, weight = store._claim(adapter_id)
        for mi, m in enumerate(store.config.target_modules):
            keys_a, keys_b = plan[mi]
            self._fold(weight.wa[m], weight.wb[m], [view(k) for k in keys_a], [view(k) for k in keys_b], rank,
                       scale)
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
        if self._file_done is not None:
            self._file_done.synchronize()  # the pinned buffer's previous contents have reached the device
        source = _TensorSource(_weights_file(path), self._file_buffer, pin=self._cuda)
        self._file_buffer = source.buffer
        key_fn = peft_key_fn(cfg.hf_config.model_type, adapter_name)
        first = key_fn(0, cfg.target_modules[0])[0]
        rank = source.shape(first)[0] if first in source else cfg.lora_rank  # _factors reports a missing key
        if rank > cfg.lora_rank or (rank < cfg.lora_rank and not (pad_rank or not strict)):
            raise ValueError(f"adapter '{adapter_id}' has rank {rank} but this store serves rank {cfg.lora_rank}"
                             + ("" if rank > cfg.lora_rank else "; pass pad_rank=True to zero-pad it into a slot"))
        scale = 1.0 if alpha is None else alpha / rank
        plan = self._factors(source, key_fn, rank, adapter_id)  # everything checked before a slot is taken
        if self._device_ready(source, plan):
            self.commit_on_device(adapter_id, source, plan, rank, scale)
            return
        index, image = self._image()
        self.stage(image, source, plan, rank, scale)
        self.commit(adapter_id, index, image)


def registrar_for(store: AdapterStore) -> AdapterRegistrar:
    """The store's registrar (created on first use; its pinned images live as long as the store)."""
    reg = getattr(store, "_registrar", None)
    if reg is None:
        reg = AdapterRegistrar(store)
        store._registrar = reg
    return reg


def peft_rank(path: str, config, adapter_name: str = "default") -> int:
    """The rank of the PEFT adapter at ``path``: its ``adapter_config.json``'s ``r``, or
    else the first target module's A in its weights file."""
    directory = path if os.path.isdir(path) else (os.path.dirname(path) or ".")
    meta = PeftAdapterConfig.read(directory)
    if meta is not None and meta.rank is not None:
        return int(meta.rank)
    source = _TensorSource(_weights_file(path))
    first = peft_key_fn(config.hf_config.model_type, adapter_name)(0, config.target_modules[0])[0]
    if first not in source:
        raise KeyError(f"the adapter at {path} has no tensor '{first}'")
    return int(source.shape(first)[0])


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
    from latefuse_b200.rank_buckets import RankBucketStore

    if isinstance(store, RankBucketStore):  # kept at its own rank, in that rank's bucket
        store.load_peft(adapter_id, path, adapter_name=adapter_name, lora_alpha=lora_alpha, strict=strict)
        return
    registrar_for(store).register(adapter_id, path, adapter_name=adapter_name, lora_alpha=lora_alpha,
                                  strict=strict, pad_rank=pad_rank)
