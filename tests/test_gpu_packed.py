"""The padding-free serving path through the public task API (real tokens only,
rows grouped by tenant), bf16 (2e-2 relative): on a tiny BERT (FlashAttention
varlen and CUDA-core LoRA: head_dim 8, rank 4) against the padded forward of the
same pipeline, and on an XLM-R-shaped encoder with head_dim 64 and rank 16
(tcgen05 attention and LoRA kernels) against the oracle."""

from __future__ import annotations

import pytest
import torch

import latefuse_b200 as lf
from tests._fixtures import insert_adapters, texts, tiny_bert_dir

pytestmark = pytest.mark.gpu


def close(a, b, tol=2e-2):
    a, b = a.float(), b.float()
    rel = ((a - b).norm(dim=-1) / b.norm(dim=-1).clamp_min(1e-6)).max().item()
    assert rel < tol, rel


def test_tiny_bert_packed_matches_padded(tmp_path, cuda):
    path, g = tiny_bert_dir(tmp_path)
    kw = dict(lora_rank=4, batch_size=8, max_seq_len=16, dtype=torch.bfloat16, device=cuda, engine="bert")
    packed = lf.MultiTenantEmbedder.from_pretrained(path, **kw)
    padded = lf.MultiTenantEmbedder.from_pretrained(path, pack_tokens=False, **kw)
    for emb in (packed, padded):
        insert_adapters(emb.store, g["adapters"], emb.config)
    assert packed.model.supports_packing
    t, ten = texts(11), ["acme", "globex", "globex"] * 3 + ["acme", "acme"]
    for pooling in ("cls", "mean", "auto"):
        close(packed.embed(t, ten, pooling=pooling), padded.embed(t, ten, pooling=pooling))
    packed.check_device_status()


def test_head_dim_64_packed_matches_oracle(cuda):
    """Ragged lengths across several 128-token tiles and tenant runs: the tcgen05
    attention and LoRA kernels on the packed layout against the oracle's
    restatement of the reference's padded forward (stock HF model + per-row bmm
    hooks) with the same weights and adapters; the padded path of this library
    is checked against the oracle the same way."""
    import torch.nn.functional as F

    from oracle.encoder import HookedEncoder
    from tests._fixtures import adapters_of, hf_model, row_rel, serving_config

    conf = dict(vocab_size=1000, hidden_size=128, num_hidden_layers=2, num_attention_heads=2, intermediate_size=512,
                max_position_embeddings=300, pad_token_id=1, type_vocab_size=1)
    base, hf = hf_model("xlmr", conf, cuda, torch.bfloat16)
    cfg = serving_config(hf, cuda, torch.bfloat16, 16, ["query", "key", "value", "dense"], 6, 256)
    model = lf.EncoderWithLora.from_hf_model(base, cfg)
    store = lf.AdapterStore(cfg, capacity=8)
    store.fill_random_(8, std=0.05, generator=torch.Generator(device=cuda).manual_seed(1))
    packed = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False)
    padded = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False, pack_tokens=False)
    assert packed.model.supports_packing and packed.model.head_dim == 64
    gen = torch.Generator().manual_seed(7)
    lengths = [256, 3, 129, 64, 200, 1]
    ids = torch.randint(5, 1000, (6, 256), generator=gen)
    ids[:, 0] = 0
    mask = torch.zeros(6, 256, dtype=torch.long)
    for b, n in enumerate(lengths):
        mask[b, :n] = 1
        ids[b, n:] = 1
    tenants = [store.adapter_ids()[i] for i in (0, 3, 3, 5, 0, 7)]
    oracle = HookedEncoder(base, adapters_of(store, tenants), cfg.target_modules)
    for pooling in ("cls", "mean"):
        ref = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, pooling).float(), dim=-1)
        for emb in (packed, padded):
            assert row_rel(emb.embed_tokens(ids, mask, tenants, pooling=pooling), ref) < 2e-2
    oracle.close()
    packed.check_device_status()
    # the streaming form (two batches in flight) returns the same rows, in batch order
    one = packed.embed_tokens(ids, mask, tenants).cpu()
    rev = packed.embed_tokens(ids.flip(0), mask.flip(0), tenants[::-1]).cpu()
    outs = list(packed.embed_tokens_stream([(ids, mask, tenants), (ids.flip(0), mask.flip(0), tenants[::-1]),
                                            (ids, mask, tenants)], depth=2))
    assert [o.is_pinned() for o in outs] == [True] * 3
    assert torch.equal(outs[0], one) and torch.equal(outs[1], rev) and torch.equal(outs[2], one)
