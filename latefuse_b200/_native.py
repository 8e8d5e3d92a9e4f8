"""ctypes binding of the C ABI in ``include/latefuse_b200.h``.

This is the only module that talks to ``liblatefuse_b200.so``.  Every compute
entry point of the package goes through it; there is no CPU or pure-PyTorch
fallback for the LoRA delta, the heads or the pooling kernels, so a missing or
unloadable library raises :class:`NativeLibraryError` instead of silently
computing something else.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p

import torch

from latefuse_b200._build import LIB_PATH

LF_OK = 0
TILE_TOKENS = 128
LF_DTYPE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
LF_POOL = {"cls": 0, "mean": 1, "none": 2}
LF_OPT_FORCE_SIMT = 1
LF_OPT_SHRINK_CLUSTER = 2
LF_OPT_REQUIRE_TC = 3
LF_OPT_PERSISTENT = 4
LF_OPT_FUSED_APPLY = 5
LF_OPT_FUSED_SPLIT = 6

LF_STATUS_BAD_SLOT, LF_STATUS_BAD_SEGMENT, LF_STATUS_TIMEOUT, LF_STATUS_BAD_HEAD = 1, 2, 4, 8

STATUS_BITS = {
    1: "segment names a slot outside the cache",
    2: "segment (or attention record) outside the token range",
    4: "on-chip wait timed out",
    8: "head rows outside the head cache",
}

#: Every symbol the header declares, with (restype, argtypes).
SIGNATURES: dict[str, tuple] = {
    "lf_version": (c_char_p, []),
    "lf_last_error": (c_char_p, []),
    "lf_device_supported": (c_int, [c_int]),
    "lf_set_option": (c_int, [c_int, c_int]),
    "lf_launch_count": (c_uint64, []),
    "lf_lora_shrink": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int64, c_int64, c_int, c_int, POINTER(c_int32),
        c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "lf_lora_shrink_blocked": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int64, c_int64, c_int, c_int, POINTER(c_int32),
        c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "lf_lora_expand": (c_int, [
        c_void_p, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int64, c_int64, c_int, c_int, POINTER(c_int32), POINTER(c_int64),
        c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p]),
    "lf_lora_workspace_bytes": (c_size_t, [c_int, c_int64, c_int, c_int]),
    "lf_lora_apply": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
        POINTER(c_int32), POINTER(c_int64), c_void_p, c_void_p, c_void_p, c_int,
        c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lf_lora_apply_into": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
        POINTER(c_int32), POINTER(c_int64), c_void_p, c_void_p, c_void_p, c_int,
        c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lf_lora_apply_noalloc": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
        POINTER(c_int32), POINTER(c_int64), c_void_p, c_void_p, c_void_p, c_int,
        c_void_p, c_int, c_int, c_void_p]),
    "lf_cache_gather": (c_int, [
        c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int, c_void_p, c_int,
        c_void_p, c_void_p]),
    "lf_cache_write_slot": (c_int, [
        c_void_p, c_void_p, c_int64, c_int, c_int, c_size_t, c_void_p, c_size_t]),
    "lf_arena_create": (c_int, [c_int, c_size_t, POINTER(c_void_p)]),
    "lf_arena_grow": (c_int, [c_void_p, c_size_t]),
    "lf_arena_base": (c_void_p, [c_void_p]),
    "lf_arena_mapped_bytes": (c_size_t, [c_void_p]),
    "lf_arena_destroy": (c_int, [c_void_p]),
    "lf_head_forward": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_int, c_int, c_int, c_int,
        c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int,
        c_void_p, c_void_p, c_void_p]),
    "lf_head_forward_rows": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
        c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "lf_linear": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int,
        c_int, c_int, c_void_p]),
    "lf_linear_accumulate": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int,
        c_int, c_void_p]),
    "lf_linear_lora": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int,
        c_int, c_int, c_void_p, c_int, c_void_p, c_int64, c_int64, c_int, c_int, POINTER(c_int32), c_int,
        c_int, c_void_p, c_void_p, c_void_p]),
    "lf_linear_lora_shrink": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_int64, c_int64, c_int,
        c_int, c_int, c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int,
        POINTER(c_int32), c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "lf_add_layernorm": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, ctypes.c_float,
        c_int64, c_int, c_void_p, c_int64]),
    "lf_embed_layernorm": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
        c_int64, c_int64, c_void_p, c_void_p, c_void_p, ctypes.c_float, c_int64, c_int, c_void_p, c_int64,
        c_void_p]),
    "lf_gelu": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int64]),
    "lf_attention_varlen": (c_int, [
        c_void_p, c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
        c_void_p, c_int, ctypes.c_float, c_void_p, c_int64, c_void_p]),
}


class NativeLibraryError(RuntimeError):
    """The native library is missing, unloadable, or a call into it failed."""


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """The loaded library (loaded on first use). Raises if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise NativeLibraryError(
                f"{LIB_PATH} is missing: build it with `python -m latefuse_b200._build` "
                "(or __graft_entry__.build()). latefuse_b200 has no non-native fallback."
            )
        try:
            handle = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != LF_OK:
        msg = lib().lf_last_error().decode(errors="replace")
        raise NativeLibraryError(f"{what} failed (code {rc}): {msg}")


def version() -> str:
    return lib().lf_version().decode()


def launch_count() -> int:
    return int(lib().lf_launch_count())


def set_option(key: int, value: int) -> None:
    check(lib().lf_set_option(key, value), "lf_set_option")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return LF_DTYPE[dtype]
    except KeyError:
        raise NativeLibraryError(f"dtype {dtype} is not supported (f32, bf16, f16)") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device; returns it. Raises on CPU tensors (no fallback)."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise NativeLibraryError(
                f"latefuse_b200 kernels need CUDA tensors; got a tensor on {t.device}. "
                "There is no CPU implementation of the serving path."
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise NativeLibraryError(f"tensors on {dev} and {t.device}")
    return dev


def i32_array(values) -> ctypes.Array:
    vals = list(values)
    return (c_int32 * max(1, len(vals)))(*vals)


def i64_array(values) -> ctypes.Array:
    vals = list(values)
    return (c_int64 * max(1, len(vals)))(*vals)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def decode_status(bits: int) -> str:
    return "; ".join(msg for bit, msg in STATUS_BITS.items() if bits & bit) or "ok"
