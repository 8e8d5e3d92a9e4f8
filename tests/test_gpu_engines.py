"""GPU parity of both engines (stock-HF hooks and the native encoder) with the
reference (golden fixtures, f32 1e-5) and with the oracle run on the same GPU in
bf16 (2e-2 relative)."""

from __future__ import annotations

import pytest
import torch

import latefuse_b200 as lf
from latefuse_b200.batch import BatchLora
from latefuse_b200.lora import SegmentTable
from oracle.encoder import HookedEncoder
from tests._fixtures import insert_adapters, tiny_xlmr

pytestmark = pytest.mark.gpu


def setup(cuda, dtype, engine):
    base, g = tiny_xlmr(dtype)
    c = lf.LoraServingConfig(model_name="tiny-xlmr", lora_rank=8, batch_size=3, max_seq_len=20,
                             target_modules=g["targets"], device=cuda, dtype=dtype, hf_config=base.config)
    store = lf.AdapterStore(c)
    insert_adapters(store, g["adapters"], c)
    if engine == "hf":
        model = lf.HFEncoderWithLora(base.to(cuda), c).eval()
    else:
        model = lf.EncoderWithLora.from_hf_model(base, c)
    return model, store, c, g


def batch_for(store, c, g, skip_padding):
    slots = store.slots(g["tenants"])
    lengths = g["mask"].sum(1).tolist() if skip_padding else None
    return BatchLora(store, SegmentTable.for_padded(slots, c.max_seq_len, c.device, lengths=lengths))


@pytest.mark.parametrize("engine", ["hf", "bert"])
@pytest.mark.parametrize("skip_padding", [False, True])
def test_f32_matches_reference_fixture(cuda, engine, skip_padding):
    model, store, c, g = setup(cuda, torch.float32, engine)
    ids, mask = g["ids"].to(cuda), g["mask"].to(cuda)
    with torch.no_grad():
        cls = model.encode_pooled(ids, mask, batch_for(store, c, g, skip_padding), pooling="cls")
        mean = model.encode_pooled(ids, mask, batch_for(store, c, g, skip_padding), pooling="mean")
        base = model.encode_pooled(ids, mask, None, apply_lora=False, pooling="cls")
    torch.testing.assert_close(cls.cpu(), g["pooled_cls"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(mean.cpu(), g["pooled_mean"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(base.cpu(), g["base_cls"], atol=1e-5, rtol=1e-5)
    assert model._runner.status.item() == 0


@pytest.mark.parametrize("engine", ["hf", "bert"])
def test_layerwise_weights_path_matches_slot_path(cuda, engine):
    model, store, c, g = setup(cuda, torch.float32, engine)
    ids, mask = g["ids"].to(cuda), g["mask"].to(cuda)
    asm = lf.IndexSelectBatchAssembler(store, c)
    with torch.no_grad():
        a = model.encode_pooled(ids, mask, asm.to_layerwise(g["tenants"]), pooling="cls")
        b = model.encode_pooled(ids, mask, batch_for(store, c, g, False), pooling="cls")
    torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("engine", ["hf", "bert"])
def test_bf16_matches_oracle_on_gpu(cuda, engine):
    model, store, c, g = setup(cuda, torch.bfloat16, engine)
    base_ref, _ = tiny_xlmr(torch.bfloat16)
    oracle = HookedEncoder(base_ref.to(cuda), g["adapters"], g["targets"])
    ids, mask = g["ids"].to(cuda), g["mask"].to(cuda)
    with torch.no_grad():
        ours = model.encode_pooled(ids, mask, batch_for(store, c, g, True), pooling="cls").float()
    ref = oracle.encode_pooled(ids, mask, g["tenants"], "cls").float()
    rel = ((ours - ref).norm(dim=-1) / ref.norm(dim=-1)).max().item()
    assert rel < 2e-2, rel
    assert (ours - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()


@pytest.mark.parametrize("pooling", ["cls", "mean", "auto"])
def test_packed_forward_matches_oracle_bf16(cuda, pooling):
    """The padding-free forward (real tokens only, rows grouped by tenant,
    attention per sequence) against the reference's padded forward run by the
    oracle on the same GPU, and against this engine's padded path."""
    model, store, c, g = setup(cuda, torch.bfloat16, "bert")
    assert model.supports_packing
    base_ref, _ = tiny_xlmr(torch.bfloat16)
    oracle = HookedEncoder(base_ref.to(cuda), g["adapters"], g["targets"])
    ids, mask = g["ids"].to(cuda), g["mask"].to(cuda)
    lengths = g["mask"].sum(1).tolist()
    pb = model.pack(g["ids"], lengths, store.slots(g["tenants"]))
    assert pb.n_tokens == sum(lengths)
    with torch.no_grad():
        ours = model.encode_pooled_packed(pb, store, pooling).float()
        padded = model.encode_pooled(ids, mask, batch_for(store, c, g, True), pooling=pooling).float()
    ref = oracle.encode_pooled(ids, mask, g["tenants"], pooling).float()
    for got in (ours, padded):
        rel = ((got - ref).norm(dim=-1) / ref.norm(dim=-1)).max().item()
        assert rel < 2e-2, rel
        assert (got - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
    assert model._runner.status.item() == 0


def test_packed_forward_tenant_isolation_and_row_order(cuda):
    """Each row's pooled output depends only on its own tokens and tenant:
    permuting rows (which changes the packed layout and segment runs) permutes
    the outputs, and a row served alone equals the same row in a mixed batch."""
    model, store, c, g = setup(cuda, torch.bfloat16, "bert")
    ids, mask, tenants = g["ids"], g["mask"], list(g["tenants"])
    lengths = mask.sum(1).tolist()
    with torch.no_grad():
        full = model.encode_pooled_packed(model.pack(ids, lengths, store.slots(tenants)), store, "cls")
        perm = list(reversed(range(len(tenants))))
        pb = model.pack(ids[perm], [lengths[i] for i in perm], store.slots([tenants[i] for i in perm]))
        permuted = model.encode_pooled_packed(pb, store, "cls")
        alone = model.encode_pooled_packed(model.pack(ids[:1], lengths[:1], store.slots(tenants[:1])), store, "cls")
    torch.testing.assert_close(permuted, full[perm], atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(alone[0], full[0], atol=2e-2, rtol=2e-2)


def test_hooks_must_all_fire(cuda):
    model, store, c, g = setup(cuda, torch.float32, "hf")
    ids, mask = g["ids"].to(cuda), g["mask"].to(cuda)
    with pytest.raises(RuntimeError, match="hooks fired"):
        # a batch whose hidden states never match the expected shape (wrong rows) skips every hook
        model._expected_shape = None
        real = model.base.forward

        def bad_forward(**kw):
            model._expected_shape = (0, 0, 0)
            return real(**kw)

        model.base.forward = bad_forward
        model.encode_pooled(ids, mask, batch_for(store, c, g, False), pooling="cls")
    model.base.forward = real


def test_closed_engine_refuses(cuda):
    model, store, c, g = setup(cuda, torch.float32, "hf")
    model.close()
    with pytest.raises(RuntimeError, match="closed"):
        model.encode_pooled(g["ids"].to(cuda), g["mask"].to(cuda), batch_for(store, c, g, False))
