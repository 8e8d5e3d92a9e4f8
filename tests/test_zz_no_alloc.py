"""lf_lora_apply_noalloc: the late-fusion delta for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc (a host framework that owns
every device allocation, or a serving loop that must not synchronise or fail on
an allocation), so they cannot provide lf_lora_apply's workspace.  The no-alloc
entry point keeps that workspace in a static device array instead.  These tests
call it through the C ABI and check it against lf_lora_apply on the same inputs,
twice in a row (the shared scratch keeps the previous call's contents), and
that an oversized batch is refused.  This file is collected last so that a run
stopping at the first failure has already run every other test.
"""

from __future__ import annotations

import pytest
import torch

from latefuse_b200 import _native as nat
from latefuse_b200.lora import FactorCache, SegmentTable, _seg_args, lora_apply, workspace_bytes

pytestmark = pytest.mark.gpu

LF_ERR_WORKSPACE = 4
SCRATCH_BYTES = 8 << 20


def inputs(dev, T=640, H=256, R=16, n_mod=3, n_slots=5, seed=0):
    g = torch.Generator().manual_seed(seed)
    cache = (torch.randn(n_slots, n_mod, 2, H * R, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    fc = FactorCache(a=cache, b=cache, a_offset=0, b_offset=H * R, a_slot_stride=cache.stride(0),
                     b_slot_stride=cache.stride(0), a_module_stride=cache.stride(1), b_module_stride=cache.stride(1),
                     n_slots=n_slots, hidden=H, rank=R)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    y = torch.randn(T, n_mod * H, generator=g).to(torch.bfloat16).to(dev)
    segs = SegmentTable([0, 200, 330], [200, 130, 300], [3, 0, 4], T, dev)
    return fc, x, y, segs


def call_noalloc(fc, x, y, segs, modules, offs, status):
    lib = nat.lib()
    rc = lib.lf_lora_apply_noalloc(
        torch.cuda.current_stream().cuda_stream, nat.dtype_code(x.dtype), x.data_ptr(), x.stride(0), y.data_ptr(),
        y.stride(0), x.shape[0], fc.hidden, fc.rank, fc.a_ptr, fc.a_slot_stride, fc.a_module_stride, fc.b_ptr,
        fc.b_slot_stride, fc.b_module_stride, fc.n_slots, len(modules), nat.i32_array(modules),
        nat.i64_array(offs), *_seg_args(segs), status.data_ptr())
    return rc


def test_noalloc_matches_allocating_entry_point(cuda):
    """Same kernels, same inputs: the no-alloc call must give the allocating call's
    bits exactly, on a first and a second call (a stale row left in the shared
    scratch by the first call would show up here), and once the array exists
    (after the first call) a further call must leave the device's free memory
    unchanged."""
    fc, x, y, segs = inputs(cuda)
    H = fc.hidden
    modules, offs = [0, 1, 2], [0, H, 2 * H]
    ws = torch.empty(workspace_bytes(x.dtype, x.shape[0], fc.rank, 3), dtype=torch.uint8, device=cuda)
    want = y.clone()
    lora_apply(x, want, fc, segs, modules, offs, ws)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = [y.clone() for _ in range(3)]
    for i, got in enumerate(outs):  # calls in a row over the same shared scratch
        if i == 2:
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info(cuda)[0]
        rc = call_noalloc(fc, x, got, segs, modules, offs, status)
        assert rc == 0, nat.lib().lf_last_error()
        torch.cuda.synchronize()
        if i == 2:
            assert torch.cuda.mem_get_info(cuda)[0] == free_before
        assert status.item() == 0
        assert not torch.equal(got, y)  # the delta is not zero
        assert torch.equal(got, want), f"call {i}: differs from lf_lora_apply"


def test_noalloc_rejects_batches_beyond_the_scratch(cuda):
    big_t = SCRATCH_BYTES // (16 * 3 * 2) + 128  # n_tokens whose shrink output exceeds the scratch
    fc, x, y, segs = inputs(cuda, T=big_t)  # real buffers of that size: nothing may be read out of bounds
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib = nat.lib()
    rc = lib.lf_lora_apply_noalloc(
        torch.cuda.current_stream().cuda_stream, nat.dtype_code(x.dtype), x.data_ptr(), x.stride(0), y.data_ptr(),
        y.stride(0), big_t, fc.hidden, fc.rank, fc.a_ptr, fc.a_slot_stride, fc.a_module_stride, fc.b_ptr,
        fc.b_slot_stride, fc.b_module_stride, fc.n_slots, 3, nat.i32_array([0, 1, 2]),
        nat.i64_array([0, fc.hidden, 2 * fc.hidden]), *_seg_args(segs), status.data_ptr())
    assert rc == LF_ERR_WORKSPACE
    assert b"static scratch" in lib.lf_last_error()
