"""The serving path at the benchmark configurations' own dimensions, against the oracle.

Every test builds one seeded random-init HuggingFace encoder, serves it through
this library's public API, and compares with the oracle's restatement of the
reference's ``HFEncoderWithLora`` (stock HF forward + per-row ``torch.bmm``
hooks, ``src/latefuse/model/hf_wrapper.py:169-219``) run on the same GPU with
the same weights and adapters:

* bge-m3 / XLM-R-large shape (H 1024, 16 heads, FFN 4096, vocab 250002), bf16,
  rank 16 on query/key/value/dense, 64 rows with lengths U[32, 512] and
  Zipf(1.1) tenants over a 2,000-slot cache, through ``embed_tokens`` on the
  padding-free path: the q/k/v projection runs on ``lf_linear_lora`` at
  (16k tokens) x 3072 x 1024 with about 33 adapter segments, exactly the
  benchmark's launch shape.  Two layers bound the runtime; every layer runs the
  same kernels.  Tolerance: 2e-2 relative per row (bf16).
* BERT-base shape (12 layers, H 768), fp32, rank 8 on query+value, 64 synthetic
  tenants, 32 x 128 rows, both engines.  Tolerance: 1e-5 max-abs (fp32).
* Classification: bge-m3 shape at rank 8 on query+value, bf16, 128 x 128 rows,
  2,000 tenants each with a head of U[2, 20] labels (coef ~ N(0, .05),
  intercept ~ N(0, .1)).  Label counts and head slicing bit-exact, probabilities
  within 2e-2.
"""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F

import latefuse_b200 as lf
from latefuse_b200.synthetic import ragged_batch, zipf_tenants
from oracle.encoder import HookedEncoder
from oracle.head import assemble_heads, head_logits, probabilities, ragged
from tests._fixtures import adapters_of, hf_model, row_rel, serving_config

pytestmark = pytest.mark.gpu

BGE_M3 = dict(vocab_size=250002, hidden_size=1024, num_attention_heads=16, intermediate_size=4096,
              max_position_embeddings=8194, pad_token_id=1, type_vocab_size=1, layer_norm_eps=1e-5)
BERT_BASE = dict(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                 intermediate_size=3072)


def test_bge_m3_shape_packed_serving_matches_oracle(cuda):
    layers, slots = 2, 2000
    base, hf = hf_model("xlmr", dict(BGE_M3, num_hidden_layers=layers), cuda, torch.bfloat16)
    cfg = serving_config(hf, cuda, torch.bfloat16, 16, ["query", "key", "value", "dense"], 64, 512)
    model = lf.EncoderWithLora.from_hf_model(base, cfg)
    store = lf.AdapterStore(cfg, capacity=slots)
    store.fill_random_(slots, std=0.02, generator=torch.Generator(device=cuda).manual_seed(1))
    emb = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False)

    ids, mask = ragged_batch(64, 512, min_len=32, max_len=512, vocab=250002, pad_id=1, cls_id=0, low_id=5, seed=3)
    tenants = [f"adapter_{int(t)}" for t in zipf_tenants(slots, 64, alpha=1.1, seed=3)]
    outs = {}
    for fused in (True, False):
        # the benchmark's path: the shrink inside the projection GEMM's launch; and the
        # shrink as its own launch before the GEMM with the delta in its accumulator
        # (that run also takes the FFN down projection on this library's GEMM)
        model.fuse_shrink = fused
        model.native_ffn_down = not fused
        model.lora_events = []
        outs[fused] = emb.embed_tokens(ids, mask, tenants)
        kinds = {k for k, _, _ in model.lora_events}
        model.lora_events = None
        emb.check_device_status()
        want = {"qkv_gemm", "dense_gemm"} | (set() if fused else {"qkv_shrink", "dense_shrink"})
        assert kinds == want, kinds
    model.fuse_shrink, model.native_ffn_down = True, False

    oracle = HookedEncoder(base, adapters_of(store, tenants), cfg.target_modules)
    ref = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "cls").float(), dim=-1)
    base_only = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "cls", apply_lora=False)
                            .float(), dim=-1)
    oracle.close()
    for fused, ours in outs.items():
        err = row_rel(ours, ref)
        assert err < 2e-2, (fused, err)
        # the adapters move the output by more than the tolerance, so a missing or
        # misrouted delta cannot pass
        assert row_rel(base_only, ref) > 2 * err


XLMR_XL = dict(vocab_size=250002, hidden_size=2560, num_attention_heads=32, intermediate_size=10240,
               max_position_embeddings=514, pad_token_id=1, type_vocab_size=1, layer_norm_eps=1e-5)


def test_xlmr_xl_shape_matches_oracle(cuda):
    """The XLM-R-XL scale-out shape (pre-LayerNorm layers, hidden 2560, 32 heads of 80,
    FFN 10240; 2 of its 36 layers) with rank 32 on query+value over 600 resident slots,
    full-length 256-token rows, through the public API (stock HF encoder, this library's
    kernels in its hooks), against the reference's per-row bmm hooks."""
    base, hf = hf_model("xlmr-xl", dict(XLMR_XL, num_hidden_layers=2), cuda, torch.bfloat16)
    cfg = serving_config(hf, cuda, torch.bfloat16, 32, ["query", "value"], 48, 256)
    model = lf.HFEncoderWithLora(base, cfg)
    store = lf.AdapterStore(cfg, capacity=600)
    store.fill_random_(600, std=0.02, generator=torch.Generator(device=cuda).manual_seed(4))
    emb = lf.MultiTenantEmbedder(cfg, engine="hf", model=model, store=store, tokenizer=False)
    ids, mask = ragged_batch(48, 256, min_len=256, max_len=256, vocab=250002, pad_id=1, cls_id=0, low_id=5, seed=4)
    tenants = [f"adapter_{int(t)}" for t in zipf_tenants(600, 48, alpha=1.1, seed=4)]
    ours = emb.embed_tokens(ids, mask, tenants).float()
    emb.check_device_status()
    oracle = HookedEncoder(base, adapters_of(store, tenants), cfg.target_modules)
    ref = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "cls").float(), dim=-1)
    base_only = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "cls", apply_lora=False)
                            .float(), dim=-1)
    oracle.close()
    err = row_rel(ours, ref)
    assert err < 2e-2, err
    assert row_rel(base_only, ref) > 2 * err


@pytest.mark.parametrize("engine", ["hf", "bert"])
def test_bert_base_f32_matches_oracle(cuda, engine):
    base, hf = hf_model("bert", BERT_BASE, cuda, torch.float32)
    cfg = serving_config(hf, cuda, torch.float32, 8, ["query", "value"], 32, 128)
    model = (lf.HFEncoderWithLora(copy.deepcopy(base), cfg) if engine == "hf"
             else lf.EncoderWithLora.from_hf_model(base, cfg))
    emb = lf.MultiTenantEmbedder(cfg, engine=engine, model=model, tokenizer=False)
    tenants_all = [f"t{i}" for i in range(64)]
    g = torch.Generator(device=cuda).manual_seed(11)
    for i, t in enumerate(tenants_all):
        emb.register_synthetic(t, seed=i)
        for m in cfg.target_modules:  # the synthetic B is zero: re-draw it so the delta is not
            emb.store.get(t).wb[m].normal_(0.0, 0.02, generator=g)
    gen = torch.Generator().manual_seed(0)
    ids = torch.randint(1000, 30522, (32, 128), generator=gen)
    mask = torch.ones(32, 128, dtype=torch.long)
    tenants = [tenants_all[int(i)] for i in torch.randint(0, 64, (32,), generator=gen)]
    ours = emb.embed_tokens(ids, mask, tenants)
    emb.check_device_status()
    oracle = HookedEncoder(base, adapters_of(emb.store, tenants), cfg.target_modules)
    ref = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "cls"), dim=-1)
    base_only = F.normalize(oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "cls", apply_lora=False),
                            dim=-1)
    oracle.close()
    err = (ours - ref).abs().max().item()
    assert err <= 1e-5, err
    assert (base_only - ref).abs().max().item() > 100 * max(err, 1e-7)


def test_bge_m3_shape_classification_matches_oracle(cuda):
    layers, n_tenants, H = 2, 2000, 1024
    base, hf = hf_model("xlmr", dict(BGE_M3, num_hidden_layers=layers), cuda, torch.bfloat16)
    cfg = serving_config(hf, cuda, torch.bfloat16, 8, ["query", "value"], 128, 128)
    model = lf.EncoderWithLora.from_hf_model(base, cfg)
    store = lf.AdapterStore(cfg, capacity=n_tenants)
    store.fill_random_(n_tenants, std=0.02, generator=torch.Generator(device=cuda).manual_seed(2),
                       prefix="tenant_")
    clf = lf.MultiTenantClassifier(cfg, engine="bert", model=model, store=store, tokenizer=False)
    g = torch.Generator().manual_seed(5)
    heads = {}
    for i in range(n_tenants):
        n = int(torch.randint(2, 21, (1,), generator=g))
        coef = torch.randn(n, H, generator=g) * 0.05
        icpt = torch.randn(n, generator=g) * 0.1
        clf.heads.load(f"tenant_{i}", coef, icpt)
        heads[f"tenant_{i}"] = (coef.to(torch.bfloat16), icpt.to(torch.bfloat16))

    ids, mask = ragged_batch(128, 128, min_len=128, max_len=128, vocab=250002, pad_id=1, cls_id=0, low_id=5,
                             seed=9)
    tenants = [f"tenant_{int(t)}" for t in zipf_tenants(n_tenants, 128, alpha=1.1, seed=9)]
    logits, probs, num_labels = clf.classify_tokens(ids, mask, tenants)
    clf.check_device_status()

    coef_ref, icpt_ref, nl_ref = assemble_heads(heads, tenants, H, torch.bfloat16)
    assert num_labels == nl_ref
    batched = clf.heads.assemble(tenants)  # the reference's padded layout, bit for bit
    assert torch.equal(batched.coef.cpu(), coef_ref) and torch.equal(batched.intercept.cpu(), icpt_ref)
    assert batched.num_labels == nl_ref

    oracle = HookedEncoder(base, adapters_of(store, tenants), cfg.target_modules)
    pooled_ref = oracle.encode_pooled(ids.to(cuda), mask.to(cuda), tenants, "auto")
    oracle.close()
    ref_logits = ragged(head_logits(pooled_ref, coef_ref.to(cuda), icpt_ref.to(cuda)).float().cpu(), nl_ref)
    ref_probs = probabilities(ref_logits)
    got_probs = [row[:n] for row, n in zip(probs.tolist(), num_labels)]
    got_logits = [row[:n] for row, n in zip(logits.float().tolist(), num_labels)]
    assert [len(r) for r in got_probs] == nl_ref
    worst = max(abs(a - b) for r1, r2 in zip(got_probs, ref_probs) for a, b in zip(r1, r2))
    assert worst <= 2e-2, worst
    scale = max(abs(v) for r in ref_logits for v in r)
    worst_logit = max(abs(a - b) for r1, r2 in zip(got_logits, ref_logits) for a, b in zip(r1, r2))
    assert worst_logit <= 2e-2 * scale, (worst_logit, scale)
    assert all(abs(sum(r) - 1.0) < 1e-4 for r in got_probs)
