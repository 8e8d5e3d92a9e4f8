"""The tcgen05 varlen attention kernel against the attention of each sequence
computed in f32 from the same half-precision q, k, v (the reference's
``softmax(q k^T * scale) @ v`` without padding), and against FlashAttention's
varlen kernel.  Tolerance: max-abs error within 2e-2 of the output's max-abs,
relative Frobenius error below 1e-2 (P and the output are rounded to the model
dtype)."""

from __future__ import annotations

import pytest
import torch

from latefuse_b200.encoder_ops import attention_varlen
from latefuse_b200.engine import varlen_attention
from latefuse_b200.packing import attention_items

pytestmark = pytest.mark.gpu


def run_case(cuda, lengths, nh, dtype, seed, key_growth=0.0):
    g = torch.Generator(device=cuda).manual_seed(seed)
    T, H = sum(lengths), nh * 64
    qkv = torch.randn(T, 3 * H, device=cuda, generator=g)
    starts = [sum(lengths[:i]) for i in range(len(lengths))]
    if key_growth:  # later keys of every sequence score higher: the running max moves between tiles
        for s0, n in zip(starts, lengths):
            pos = torch.arange(n, device=cuda, dtype=torch.float32)
            qkv[s0:s0 + n, H:2 * H] *= (1 + key_growth * pos / 128).unsqueeze(1)
    qkv = qkv.to(dtype)
    items = torch.tensor(attention_items(starts, lengths), dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.full((T, H), float("nan"), device=cuda, dtype=dtype)
    attention_varlen(qkv, nh, items, 64 ** -0.5, out=out, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    assert not out.isnan().any(), "a row was not written"
    q, k, v = qkv.float().view(T, 3, nh, 64).unbind(1)
    ref = torch.empty(T, nh, 64, device=cuda)
    for s0, n in zip(starts, lengths):
        sc = torch.einsum("ihd,jhd->hij", q[s0:s0 + n], k[s0:s0 + n]) * 64 ** -0.5
        ref[s0:s0 + n] = torch.einsum("hij,jhd->ihd", sc.softmax(-1), v[s0:s0 + n])
    ref = ref.view(T, H)
    return out, ref, qkv, starts


def check(out, ref):
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ragged_lengths(cuda, dtype):
    # last tiles of 1..128 rows: every 32-row warp and 64-key half boundary, either side
    lengths = [1, 7, 128, 129, 300, 512, 64, 33, 255, 256, 257, 65, 96, 97, 160, 161, 192, 193, 224, 225, 31, 32]
    out, ref, _, _ = run_case(cuda, lengths, 16, dtype, seed=1)
    check(out, ref)


def test_long_sequences_and_moving_max(cuda):
    """Up to 9 key tiles per sequence, with scores growing along the keys so the
    running max is raised and O rescaled in TMEM."""
    lengths = [1100, 640, 130, 5]
    out, ref, _, _ = run_case(cuda, lengths, 4, torch.bfloat16, seed=2, key_growth=3.0)
    check(out, ref)


def test_bench_shaped_batch_matches_flash_varlen(cuda):
    """64 sequences of U[32, 512] tokens, 16 heads: every CTA loops over many
    (query tile, head) units; the result agrees with FlashAttention's varlen."""
    gen = torch.Generator().manual_seed(3)
    lengths = torch.randint(32, 513, (64,), generator=gen).tolist()
    out, ref, qkv, starts = run_case(cuda, lengths, 16, torch.bfloat16, seed=3)
    check(out, ref)
    T = sum(lengths)
    cu = torch.tensor([0] + [sum(lengths[:i + 1]) for i in range(len(lengths))], dtype=torch.int32, device=cuda)
    q, k, v = qkv.view(T, 3, 16, 64).unbind(1)
    fa = varlen_attention(q, k, v, cu, max(lengths)).reshape(T, 1024)
    check(out, fa.float())


def test_rejects_unsupported_head_dim(cuda):
    from latefuse_b200 import _native as nat

    qkv = torch.zeros(16, 3 * 256, device=cuda, dtype=torch.bfloat16)
    items = torch.tensor([[0, 16, 0, 0]], dtype=torch.int32, device=cuda)
    with pytest.raises(nat.NativeLibraryError, match="head_dim"):
        attention_varlen(qkv, 2, items, 1.0)  # head_dim 128


def test_records_outside_the_batch_store_nothing(cuda):
    """A record past the last token, one with a negative start and one with a q-tile
    past its length set LF_STATUS_BAD_SEGMENT and write no row; a zero-length record
    writes nothing; the valid records are still exact."""
    from latefuse_b200 import _native as nat

    lengths = [200, 77, 129]
    T, H, nh = sum(lengths), 256, 4
    g = torch.Generator(device=cuda).manual_seed(5)
    qkv = torch.randn(T, 3 * H, device=cuda, generator=g).to(torch.bfloat16)
    starts = [0, 200, 277]
    good = torch.tensor(attention_items(starts, lengths), dtype=torch.int32)
    bad = torch.tensor([[T - 10, 50, 0, 0], [-1, 3, 0, 0], [200, 77, 1, 0], [5, 0, 0, 0]], dtype=torch.int32)
    items = torch.cat([good, bad]).to(cuda)
    big = torch.full((T + 256, H), 7.0, device=cuda, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    attention_varlen(qkv, nh, items, 64 ** -0.5, out=big[:T], status=status)
    torch.cuda.synchronize()
    assert status.item() & nat.LF_STATUS_BAD_SEGMENT
    assert (big[T:] == 7.0).all(), "a row past the batch was written"
    q, k, v = qkv.float().view(T, 3, nh, 64).unbind(1)
    for s0, n in zip(starts, lengths):
        sc = torch.einsum("ihd,jhd->hij", q[s0:s0 + n], k[s0:s0 + n]) * 64 ** -0.5
        ref = torch.einsum("hij,jhd->ihd", sc.softmax(-1), v[s0:s0 + n]).reshape(n, H)
        check(big[s0:s0 + n], ref)


def test_rejects_int64_records_and_wrong_out(cuda):
    qkv = torch.zeros(16, 3 * 256, device=cuda, dtype=torch.bfloat16)
    items = torch.tensor([[0, 16, 0, 0]], dtype=torch.int64, device=cuda)
    with pytest.raises(ValueError, match="int32"):
        attention_varlen(qkv, 4, items, 1.0)
    with pytest.raises(ValueError, match="out must be"):
        attention_varlen(qkv, 4, items.int(), 1.0, out=torch.empty(8, 256, device=cuda, dtype=torch.bfloat16))
