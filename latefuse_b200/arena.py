"""Growable device arena for the adapter slot cache.

The arena reserves a large range of device virtual addresses once and maps
physical memory into it on demand (``lf_arena_*``, CUDA virtual memory
management), so the cache can grow one registration at a time without ever
moving: every tensor view handed out earlier stays valid, and growth never
needs a second copy of the cache in memory.  The reference instead re-packs the
whole store into fresh tensors on the next batch after every registration
(``src/latefuse/tasks/base.py:181-190``, ``src/latefuse/weights/batch.py:163-170``),
which transiently doubles the cache's footprint.
"""

from __future__ import annotations

import ctypes

import torch

from latefuse_b200 import _native as nat


class _CudaBytes:
    """Exposes ``nbytes`` of device memory at ``ptr`` through ``__cuda_array_interface__``
    and keeps the owning arena alive for as long as a tensor views it."""

    def __init__(self, owner, ptr: int, nbytes: int):
        self._owner = owner
        self.__cuda_array_interface__ = {
            "shape": (nbytes,),
            "typestr": "|u1",
            "data": (ptr, False),
            "version": 3,
            "strides": None,
            "stream": None,
        }


class DeviceArena:
    """A contiguous, growable byte range of device memory on one GPU."""

    def __init__(self, device: torch.device, reserve_bytes: int):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DeviceArena needs a CUDA device")
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", idx)
        handle = ctypes.c_void_p()
        nat.check(nat.lib().lf_arena_create(idx, int(reserve_bytes), ctypes.byref(handle)), "lf_arena_create")
        self._handle = handle
        self.reserved = int(reserve_bytes)

    @property
    def base(self) -> int:
        return int(nat.lib().lf_arena_base(self._handle) or 0)

    @property
    def mapped_bytes(self) -> int:
        return int(nat.lib().lf_arena_mapped_bytes(self._handle))

    def grow(self, nbytes: int) -> None:
        """Ensure at least ``nbytes`` are mapped (the base address never changes)."""
        nat.check(nat.lib().lf_arena_grow(self._handle, int(nbytes)), "lf_arena_grow")

    def tensor(self, nbytes: int | None = None) -> torch.Tensor:
        """A uint8 tensor viewing the first ``nbytes`` mapped bytes (default: all)."""
        n = self.mapped_bytes if nbytes is None else int(nbytes)
        if n > self.mapped_bytes:
            raise ValueError(f"{n} bytes requested but only {self.mapped_bytes} mapped")
        with torch.cuda.device(self.device):
            return torch.as_tensor(_CudaBytes(self, self.base, n), device=self.device)

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            try:
                nat.lib().lf_arena_destroy(h)
            except Exception:
                pass
            self._handle = None
