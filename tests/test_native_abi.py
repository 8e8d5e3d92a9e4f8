"""The C ABI: the library loads, exports exactly what the header declares, and
rejects bad arguments with error codes before touching a GPU (CPU-only test)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from latefuse_b200 import _native as nat
from latefuse_b200._build import HEADER, LIB_PATH, build

LF_ERR_INVALID = 1


def header_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lf_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build()  # no-op when up to date; nvcc cross-compiles without a GPU
    return nat.lib()


def test_header_declares_the_path():
    names = header_functions()
    for required in ["lf_lora_shrink", "lf_lora_expand", "lf_lora_apply", "lf_head_forward", "lf_cache_gather",
                     "lf_cache_write_slot", "lf_arena_create", "lf_last_error"]:
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (lf_[a-z0-9_]+)", out.stdout))
    declared = set(header_functions())
    assert declared <= exported, sorted(declared - exported)
    assert declared == set(nat.SIGNATURES), "ctypes bindings out of sync with the header"
    for name in declared:
        assert getattr(lib, name) is not None


def test_version_and_options(lib):
    assert "sm_100a" in nat.version()
    assert lib.lf_set_option(999, 1) == LF_ERR_INVALID
    assert b"unknown option" in lib.lf_last_error()
    assert lib.lf_set_option(nat.LF_OPT_SHRINK_CLUSTER, 3) == LF_ERR_INVALID
    # the one-launch lf_lora_apply: 0 off, 1 one-module calls (default), 2 every module count
    for v in (0, 2, 1):
        assert lib.lf_set_option(nat.LF_OPT_FUSED_APPLY, v) == 0
    assert lib.lf_set_option(nat.LF_OPT_FUSED_APPLY, 3) == LF_ERR_INVALID
    assert b"LF_OPT_FUSED_APPLY" in lib.lf_last_error()
    for v in (4, 1, 0):  # column chunks per tile record, 0 = automatic
        assert lib.lf_set_option(nat.LF_OPT_FUSED_SPLIT, v) == 0
    assert lib.lf_set_option(nat.LF_OPT_FUSED_SPLIT, 17) == LF_ERR_INVALID
    assert lib.lf_set_option(nat.LF_OPT_FUSED_SPLIT, -1) == LF_ERR_INVALID


def test_argument_validation_happens_before_any_device_work(lib):
    mods = nat.i32_array([0])
    offs = nat.i64_array([0])
    # unknown dtype
    rc = lib.lf_lora_shrink(None, 7, None, 64, 128, 64, 16, None, 0, 0, 1, 1, mods, None, None, None, 0, None, 0, 0,
                            None, None)
    assert rc == LF_ERR_INVALID and b"dtype" in lib.lf_last_error()
    # too many modules
    rc = lib.lf_lora_expand(None, 1, None, None, 64, 128, 64, 16, None, 0, 0, 1, 5, mods, offs, None, None, None, 0,
                            None, 0, 0, 1, None)
    assert rc == LF_ERR_INVALID and b"n_modules" in lib.lf_last_error()
    # workspace too small is its own error code
    buf = ctypes.create_string_buffer(64)
    addr = ctypes.addressof(buf)
    rc = lib.lf_lora_apply(None, 1, addr, 64, addr, 64, 128, 64, 16, addr, 0, 0, addr, 0, 0, 1, 1, mods, offs,
                           None, None, None, 0, None, 0, 0, addr, 16, None)
    assert rc == 4 and b"workspace" in lib.lf_last_error()
    # bad tile list
    rc = lib.lf_lora_apply(None, 1, addr, 64, addr, 64, 128, 64, 16, addr, 0, 0, addr, 0, 0, 1, 1, mods, offs,
                           None, None, None, 0, None, 3, 0, addr, 1 << 20, None)
    assert rc == LF_ERR_INVALID and b"tile" in lib.lf_last_error()
    # head: unknown pooling
    rc = lib.lf_head_forward(None, 1, addr, 64, 64, None, 2, 4, 64, 9, None, None, None, None, 0, None, None, 0,
                             None, None, None)
    assert rc == LF_ERR_INVALID and b"pooling" in lib.lf_last_error()
    # cache write out of range
    rc = lib.lf_cache_write_slot(None, addr, 64, 5, 4, 0, addr, 16)
    assert rc == LF_ERR_INVALID
    # layernorm: hidden not a multiple of 8; gelu: size not a multiple of 8
    rc = lib.lf_add_layernorm(None, 1, addr, 12, None, 0, None, addr, addr, 1e-5, 4, 12, addr, 12)
    assert rc == LF_ERR_INVALID and b"multiple of 8" in lib.lf_last_error()
    rc = lib.lf_gelu(None, 1, addr, addr, 7)
    assert rc == LF_ERR_INVALID and b"multiple of 8" in lib.lf_last_error()
    # layernorm: a second matrix and a row vector together
    rc = lib.lf_add_layernorm(None, 1, addr, 16, addr, 16, addr, addr, addr, 1e-5, 4, 16, addr, 16)
    assert rc == LF_ERR_INVALID and b"together" in lib.lf_last_error()


def test_workspace_size(lib):
    assert lib.lf_lora_workspace_bytes(1, 1000, 16, 3) == (1000 * 16 * 3 * 2 + 255) // 256 * 256
    assert lib.lf_lora_workspace_bytes(0, 10, 8, 1) == 512
    assert lib.lf_lora_workspace_bytes(1, 0, 8, 1) == 0


def test_package_has_no_path_to_the_oracle():
    """The product never imports the oracle (it is test infrastructure)."""
    pkg = Path(nat.__file__).resolve().parent
    for py in pkg.rglob("*.py"):
        src = py.read_text()
        assert "import oracle" not in src and "from oracle" not in src, py
