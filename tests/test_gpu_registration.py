"""Registration of PEFT adapter files into the slot cache on the GPU, and mixed-rank serving.

* A ``.safetensors`` adapter goes to the device in one copy and is folded there;
  a ``.bin`` adapter is folded on the host into a pinned slot image.  Both must
  leave exactly the bits of the reference's ``LoraWeight.copy_from_tensors``
  (cast to bf16, transpose, multiply by alpha / r in bf16;
  ``src/latefuse/weights/store.py:51-56``).
* A rank-8 adapter zero-padded into a rank-16 store (``pad_rank=True``) serves,
  through the tcgen05 shrink and the projection GEMM with the delta, the same
  embeddings as the oracle's restatement of the reference forward given the
  unpadded rank-8 factors (``tests/test_mixed_rank_padding.py:56-93`` of the
  reference states the identity), within the bf16 tolerance of 2e-2.
"""

from __future__ import annotations

import json

import pytest
import torch
import torch.nn.functional as F

import latefuse_b200 as lf
from oracle.encoder import HookedEncoder
from tests._fixtures import hf_model, row_rel, serving_config

pytestmark = pytest.mark.gpu

TARGETS = ["query", "key", "value", "dense"]


def peft_dir(path, layers, hidden, rank, alpha, seed, fmt="safetensors"):
    """A PEFT adapter directory: A (r, H) and B (H, r) per layer and target, f32."""
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    key_fn = lf.peft_key_fn("xlm-roberta")
    sd = {}
    for layer in range(layers):
        for m in TARGETS:
            ka, kb = key_fn(layer, m)
            sd[ka] = torch.randn(rank, hidden, generator=g) * 0.05
            sd[kb] = torch.randn(hidden, rank, generator=g) * 0.05
    path.mkdir(parents=True)
    if fmt == "safetensors":
        save_file(sd, str(path / "adapter_model.safetensors"))
    else:
        torch.save(sd, path / "adapter_model.bin")
    (path / "adapter_config.json").write_text(json.dumps({"r": rank, "lora_alpha": alpha,
                                                         "target_modules": TARGETS}))
    return sd


def reference_fold(sd, layers, rank, alpha, module):
    """The reference's slot contents for one module: (L, H, r) A and (L, r, H) B in bf16."""
    key_fn = lf.peft_key_fn("xlm-roberta")
    a = torch.stack([sd[key_fn(i, module)[0]] for i in range(layers)])
    b = torch.stack([sd[key_fn(i, module)[1]] for i in range(layers)])
    wa = a.to(torch.bfloat16).transpose(1, 2)
    wb = b.to(torch.bfloat16).transpose(1, 2)
    return wa, wb.mul_(alpha / rank) if alpha != rank else wb


def small_pipeline(cuda, rank=16, layers=2, hidden=256):
    conf = dict(vocab_size=1000, hidden_size=hidden, num_hidden_layers=layers, num_attention_heads=hidden // 64,
                intermediate_size=4 * hidden, max_position_embeddings=600, pad_token_id=1, type_vocab_size=1)
    base, hf = hf_model("xlmr", conf, cuda, torch.bfloat16)
    cfg = serving_config(hf, cuda, torch.bfloat16, rank, TARGETS, 8, 512)
    model = lf.EncoderWithLora.from_hf_model(base, cfg)
    emb = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, tokenizer=False)
    return base, cfg, emb


@pytest.mark.parametrize("fmt", ["safetensors", "bin"])
def test_registered_slots_hold_the_reference_fold(tmp_path, cuda, fmt):
    _, cfg, emb = small_pipeline(cuda)
    sds = {}
    for i, alpha in enumerate((16, 32, 8)):
        sds[f"t{i}"] = (peft_dir(tmp_path / f"a{i}", cfg.num_layers, cfg.hidden_size, 16, alpha, seed=i, fmt=fmt),
                        alpha)
        emb.register_adapter(f"t{i}", str(tmp_path / f"a{i}"))
    emb.register_adapter("t0", str(tmp_path / "a1"))  # re-registration overwrites the tenant's slot
    sds["t0"] = sds["t1"]
    torch.cuda.synchronize()
    for t, (sd, alpha) in sds.items():
        w = emb.store.get(t)
        for m in TARGETS:
            wa, wb = reference_fold(sd, cfg.num_layers, 16, alpha, m)
            assert torch.equal(w.wa[m].cpu(), wa), (t, m)
            assert torch.equal(w.wb[m].cpu(), wb), (t, m)


def test_padded_lower_rank_adapter_serves_like_the_oracle(tmp_path, cuda):
    base, cfg, emb = small_pipeline(cuda, rank=16)
    sd8 = peft_dir(tmp_path / "r8", cfg.num_layers, cfg.hidden_size, 8, 24, seed=3)
    sd16 = peft_dir(tmp_path / "r16", cfg.num_layers, cfg.hidden_size, 16, 16, seed=4)
    with pytest.raises(ValueError, match="rank"):
        emb.register_adapter("low", str(tmp_path / "r8"))  # one rank per pipeline unless padding is asked for
    emb.register_adapter("low", str(tmp_path / "r8"), pad_rank=True)
    emb.register_adapter("full", str(tmp_path / "r16"))
    w = emb.store.get("low")
    for m in TARGETS:
        assert (w.wa[m][:, :, 8:] == 0).all() and (w.wb[m][:, 8:, :] == 0).all()

    adapters = {"low": {"wa": {}, "wb": {}}, "full": {"wa": {}, "wb": {}}}
    for m in TARGETS:  # the oracle serves the unpadded factors
        adapters["low"]["wa"][m], adapters["low"]["wb"][m] = reference_fold(sd8, cfg.num_layers, 8, 24, m)
        adapters["full"]["wa"][m], adapters["full"]["wb"][m] = reference_fold(sd16, cfg.num_layers, 16, 16, m)
    gen = torch.Generator().manual_seed(5)
    lengths = [512, 300, 129, 40, 500, 7, 256, 90]
    ids = torch.randint(5, 1000, (8, 512), generator=gen)
    ids[:, 0] = 0
    mask = (torch.arange(512).unsqueeze(0) < torch.tensor(lengths).unsqueeze(1)).long()
    ids = torch.where(mask.bool(), ids, torch.ones_like(ids))
    tenants = ["low", "full", "low", "low", "full", "full", "low", "full"]
    emb.model.lora_events = []
    ours = emb.embed_tokens(ids, mask, tenants)
    kinds = {k for k, _, _ in emb.model.lora_events}
    emb.model.lora_events = None
    emb.check_device_status()
    assert "qkv_gemm" in kinds  # the tcgen05 path, not the CUDA-core fallback
    # the reference serves one rank per batch, so the oracle runs each tenant's rows
    # on their own (rows are independent: each attends only to itself)
    oracle = HookedEncoder(base, adapters, TARGETS)
    for t in ("low", "full"):
        rows = [i for i, x in enumerate(tenants) if x == t]
        ref = F.normalize(oracle.encode_pooled(ids[rows].to(cuda), mask[rows].to(cuda), [t] * len(rows), "cls")
                          .float(), dim=-1)
        assert row_rel(ours[rows], ref) < 2e-2, t
    oracle.close()


def test_native_rank_buckets_serve_like_the_padded_store(tmp_path, cuda):
    """Rank 4, 8 and 16 PEFT adapters kept at their own ranks (RankBucketStore) and
    padded per batch: the packed forward gives the same bits as the same adapters
    zero-padded into one rank-16 store, and matches the oracle's unpadded forward;
    a following batch that puts a lower-rank tenant in a staging slot a rank-16 tenant
    held gets no trace of it."""
    from latefuse_b200.rank_buckets import RankBucketStore

    base, cfg, emb_pad = small_pipeline(cuda, rank=16)
    fleet = RankBucketStore(cfg)
    emb = lf.MultiTenantEmbedder(cfg, engine="bert", model=emb_pad.model, store=fleet, tokenizer=False)
    sds = {}
    for t, r, alpha, seed in (("r4", 4, 8, 11), ("r8", 8, 24, 12), ("r16", 16, 16, 13)):
        sds[t] = (peft_dir(tmp_path / t, cfg.num_layers, cfg.hidden_size, r, alpha, seed=seed), r, alpha)
        emb.register_adapter(t, str(tmp_path / t))
        emb_pad.register_adapter(t, str(tmp_path / t), pad_rank=True)
    assert [fleet.rank_of(t) for t in ("r4", "r8", "r16")] == [4, 8, 16]
    assert fleet.memory_bytes() * 48 == emb_pad.store.memory_bytes() * 28

    gen = torch.Generator().manual_seed(6)
    lengths = [400, 33, 257, 128, 7, 300]
    ids = torch.randint(5, 1000, (6, 512), generator=gen)
    ids[:, 0] = 0
    mask = (torch.arange(512).unsqueeze(0) < torch.tensor(lengths).unsqueeze(1)).long()
    ids = torch.where(mask.bool(), ids, torch.ones_like(ids))
    for tenants in (["r16", "r8", "r16", "r4", "r8", "r4"], ["r4", "r4", "r8", "r8", "r4", "r8"]):
        ours = emb.embed_tokens(ids, mask, tenants)
        pad = emb_pad.embed_tokens(ids, mask, tenants)
        emb.check_device_status()
        assert torch.equal(ours, pad), tenants
    adapters = {t: {"wa": {}, "wb": {}} for t in sds}
    for t, (sd, r, alpha) in sds.items():
        for m in TARGETS:
            adapters[t]["wa"][m], adapters[t]["wb"][m] = reference_fold(sd, cfg.num_layers, r, alpha, m)
    oracle = HookedEncoder(base, adapters, TARGETS)
    for t in ("r4", "r8"):
        rows = [i for i, x in enumerate(tenants) if x == t]
        ref = F.normalize(oracle.encode_pooled(ids[rows].to(cuda), mask[rows].to(cuda), [t] * len(rows), "cls")
                          .float(), dim=-1)
        assert row_rel(ours[rows], ref) < 2e-2, t
    oracle.close()
