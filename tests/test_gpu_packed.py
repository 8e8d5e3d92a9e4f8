"""The padding-free serving path through the public task API: packed forward
(real tokens only, rows grouped by tenant) against the padded forward of the
same pipeline, bf16 (2e-2 relative), on a tiny BERT (FlashAttention varlen and
CUDA-core LoRA: head_dim 8, rank 4) and on an XLM-R-shaped encoder with
head_dim 64 and rank 16 (tcgen05 attention and LoRA kernels)."""

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


def _xlmr_pipeline(cuda, pack: bool, seed: int = 0):
    from transformers import XLMRobertaConfig

    hf = XLMRobertaConfig(vocab_size=1000, hidden_size=128, num_hidden_layers=2, num_attention_heads=2,
                          intermediate_size=512, max_position_embeddings=300, pad_token_id=1, type_vocab_size=1)
    cfg = lf.LoraServingConfig(model_name="xlmr-hd64", lora_rank=16, batch_size=6, max_seq_len=256,
                               target_modules=["query", "key", "value", "dense"], device=cuda, dtype=torch.bfloat16,
                               hf_config=hf)
    model = lf.EncoderWithLora.random_init(hf, cfg, seed=seed)
    store = lf.AdapterStore(cfg, capacity=8)
    store.fill_random_(8, std=0.05, generator=torch.Generator(device=cuda).manual_seed(seed + 1))
    return lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False, pack_tokens=pack)


def test_head_dim_64_packed_matches_padded(cuda):
    """Ragged lengths across several 128-token tiles and tenant runs: the tcgen05
    attention and the persistent LoRA kernels on the packed layout agree with
    the padded forward (SDPA with a mask)."""
    packed, padded = _xlmr_pipeline(cuda, True), _xlmr_pipeline(cuda, False)
    assert packed.model.supports_packing and packed.model.head_dim == 64
    gen = torch.Generator().manual_seed(7)
    lengths = [256, 3, 129, 64, 200, 1]
    ids = torch.randint(5, 1000, (6, 256), generator=gen)
    ids[:, 0] = 0
    mask = torch.zeros(6, 256, dtype=torch.long)
    for b, n in enumerate(lengths):
        mask[b, :n] = 1
        ids[b, n:] = 1
    tenants = [packed.store.adapter_ids()[i] for i in (0, 3, 3, 5, 0, 7)]
    for pooling in ("cls", "mean"):
        a = packed.embed_tokens(ids, mask, tenants, pooling=pooling)
        b = padded.embed_tokens(ids, mask, tenants, pooling=pooling)
        close(a, b)
    packed.check_device_status()
