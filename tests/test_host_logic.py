"""Host-side logic on the CPU: stores, assemblers, heads, loaders, batching, segment tables.

Mirrors the reference's own CPU tests (``tests/test_weights.py``,
``tests/test_tasks.py`` sections 1, 5, 8, 9) for the parts that involve no kernel:
the serving path itself only runs on the GPU.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch
from transformers import BertConfig

import latefuse_b200 as lf
from latefuse_b200.batch import BatchAssembler, IndexSelectBatchAssembler
from latefuse_b200.lora import SegmentTable
from latefuse_b200.tasks import chunk_and_pad, right_padded_lengths

GOLD = Path(__file__).resolve().parent / "golden"
TINY = dict(vocab_size=100, hidden_size=32, num_hidden_layers=2, num_attention_heads=4, intermediate_size=64,
            max_position_embeddings=64, pad_token_id=0)


def cfg(rank=4, dtype=torch.float32, targets=("query", "value")):
    return lf.LoraServingConfig(model_name="tiny", lora_rank=rank, batch_size=4, max_seq_len=16,
                                target_modules=list(targets), device=torch.device("cpu"), dtype=dtype,
                                hf_config=BertConfig(**TINY))


# ---------------------------------------------------------------- batching ---
def test_chunk_and_pad_matches_reference_cases():
    cases = json.loads((GOLD / "chunking.json").read_text())
    for key, want in cases.items():
        n, bs = map(int, key.split("_"))
        assert [[c, k] for c, k in chunk_and_pad(list(range(n)), bs)] == want
    with pytest.raises(ValueError, match="must be positive"):
        list(chunk_and_pad([1], 0))


def test_pair_tiles_merge_the_halves_of_each_256_token_tile():
    from latefuse_b200.lora import _pair_tiles

    # segments [0,100) [100,300) [300,700) [700,710) over 710 tokens: 128-token tiles 0..5
    got = _pair_tiles([0, 100, 300, 700], [100, 200, 400, 10], [5, 6, 7, 8], 710)
    assert got[:4] == [0, 2, 4, 6]
    entries = [got[4 + 3 * i: 7 + 3 * i] for i in range(6)]
    assert entries == [[0, 5, 1], [1, 6, 3], [1, 6, 1], [2, 7, 3], [2, 7, 3], [3, 8, 2]]
    assert _pair_tiles([0, 5], [0, 0], [1, 2], 300) == [0, 0, 0]  # empty segments are left out


def test_right_padded_lengths():
    m = torch.tensor([[1, 1, 1, 0], [1, 0, 0, 0], [1, 1, 1, 1]])
    assert right_padded_lengths(m) == [3, 1, 4]
    assert right_padded_lengths(torch.tensor([[0, 1, 1, 1]])) is None  # left padding is not a suffix


def test_segment_table_layout_and_tiles():
    st = SegmentTable.for_padded([5, 0, 5], 200, "cpu", lengths=[200, 10, 0])
    h = st.host.tolist()
    # tile records first (16-byte aligned): {tile, first segment, count, slot of first}
    # [0,200) -> tiles 0,1 ; [200,210) -> tile 1 ; the empty segment -> none
    assert st.n_tiles == 2 and st.n_multi == 1
    assert h[:8] == [0, 0, 1, 5, 1, 0, 2, 5]
    assert h[8:11] == [0, 200, 400] and h[11:14] == [200, 10, 0] and h[14:17] == [5, 0, 5]
    assert st.real_tokens == 210
    s, l, k, t, nt, nm = st.ptrs()
    assert (t - st.table.data_ptr()) == 0 and s - t == 32 and nt == 2 and nm == 1
    # several short segments in one tile: single-segment tiles are listed first
    st2 = SegmentTable([0, 10, 130], [10, 100, 5], [1, 2, 3], 200, "cpu")
    assert st2.host.tolist()[:8] == [1, 2, 1, 3, 0, 0, 2, 1] and st2.n_multi == 1


# ------------------------------------------------------------ adapter store ---
def test_pack_rows_layout():
    """Packed order = rows sorted by slot (stable); every index table agrees with
    the padded rows; adjacent rows of one slot form one LoRA segment."""
    from latefuse_b200.packing import pack_rows

    B, S = 4, 6
    ids = torch.arange(B * S).view(B, S) + 100
    ids[0, 2] = 1  # a pad id inside a real span keeps the RoBERTa rule honest
    tt = torch.zeros(B, S, dtype=torch.long)
    tt[:, 3:] = 1
    lengths, slots = [6, 2, 4, 1], [5, 3, 5, 3]
    m = ids.ne(1).long()
    pos = torch.cumsum(m, 1) * m + 1  # HF create_position_ids_from_input_ids with pad 1
    pb = pack_rows(ids, lengths, slots, 1, tt, torch.device("cpu"))
    assert pb.order == [1, 3, 0, 2]
    assert pb.n_tokens == 13 and pb.max_len == 6
    assert pb.cu_seqlens.tolist() == [0, 2, 3, 9, 13]
    assert pb.ids.tolist() == torch.cat([ids[b, :lengths[b]] for b in pb.order]).tolist()
    assert pb.positions.tolist() == torch.cat([pos[b, :lengths[b]] for b in pb.order]).tolist()
    assert pb.token_types.tolist() == torch.cat([tt[b, :lengths[b]] for b in pb.order]).tolist()
    for b in range(B):  # first token of each input row is its CLS
        assert pb.ids[pb.first_token[b]].item() == ids[b, 0].item()
    assert pb.row_of_token.tolist() == sum(([b] * lengths[b] for b in pb.order), [])
    assert pb.row_lengths.tolist() == lengths
    segs = pb.segments
    assert segs.n_segs == 2 and segs.slots == [3, 5]
    n = segs.n_segs
    starts, seg_lens = segs.host[4 * segs.n_tiles:4 * segs.n_tiles + 3 * n].view(3, -1)[:2].tolist()
    assert starts == [0, 3] and seg_lens == [3, 10]
    # per-256-token-tile {segment, slot, halves} entries after the segment arrays: one
    # tile, both segments in its first 128-token half
    assert segs.host[4 * segs.n_tiles + 3 * n:].tolist() == [0, 2, 0, 3, 1, 1, 5, 1]
    # attention work list: one record per (sequence, 128-query tile)
    assert pb.attn_items.tolist() == [[0, 2, 0, 0], [2, 1, 0, 0], [3, 6, 0, 0], [9, 4, 0, 0]]
    arange = pack_rows(ids, lengths, slots, None, None, torch.device("cpu"))  # BERT numbering
    assert arange.positions.tolist() == torch.cat([torch.arange(lengths[b]) for b in pb.order]).tolist()
    with pytest.raises(ValueError):
        pack_rows(ids, [6, 0, 4, 1], slots, None, None, torch.device("cpu"))


def test_attention_items_order_and_tiles():
    from latefuse_b200.packing import attention_items

    items = attention_items([0, 5, 305], [5, 300, 129]).tolist()
    # the 300-token sequence (3 query tiles) first, then the 129-token one (2), then the short one
    assert items == [[5, 300, 0, 0], [5, 300, 1, 0], [5, 300, 2, 0], [305, 129, 0, 0], [305, 129, 1, 0],
                     [0, 5, 0, 0]]


def test_store_shapes_and_accounting():
    c = cfg()
    store = lf.AdapterStore(c)
    store.load_synthetic("a0", seed=0)
    store.load_synthetic("a1", seed=1)
    L, H, R = c.num_layers, c.hidden_size, c.lora_rank
    w = store.get("a0")
    for m in c.target_modules:
        assert w.wa[m].shape == (L, H, R) and w.wa[m].is_contiguous()
        assert w.wb[m].shape == (L, R, H) and w.wb[m].is_contiguous()
    assert store.memory_bytes() == len(c.target_modules) * 2 * (L * H * R * 4) * 2
    assert not torch.equal(store.get("a0").wa["query"], store.get("a1").wa["query"])


def test_store_synthetic_draws_match_reference_fixture():
    g = torch.load(GOLD / "synthetic_rng.pt", weights_only=False)
    store = lf.AdapterStore(cfg())
    store.load_synthetic("a", seed=g["seed"])
    for m in g["wa"]:
        assert torch.equal(store.get("a").wa[m], g["wa"][m])
        assert torch.equal(store.get("a").wb[m], g["wb"][m])


def test_store_errors_name_the_adapter():
    store = lf.AdapterStore(cfg())
    with pytest.raises(KeyError, match="not found"):
        store.get("nonexistent")
    with pytest.raises(KeyError, match="nobody"):
        store.slots(["nobody"])
    with pytest.raises(KeyError, match="not resident"):
        store.evict("ghost")


def test_store_slot_reuse_and_growth_keeps_views_valid():
    store = lf.AdapterStore(cfg(), capacity=2)
    for i in range(5):  # grows past the initial capacity
        store.load_synthetic(f"t{i}", seed=i)
    w1 = store.get("t1")
    before = w1.wa["query"].clone()
    for i in range(5, 40):
        store.load_synthetic(f"t{i}", seed=i)
    assert torch.equal(store.get("t1").wa["query"], before)
    assert store.get("t1") is w1
    slot3 = store.slot_of("t3")
    store.evict("t3")
    store.load_synthetic("new", seed=99)
    assert store.slot_of("new") == slot3  # freed slot is reused
    assert store.adapter_ids()[-1] == "new" and "t3" not in store


def test_store_insert_aliases_the_slot():
    c = cfg()
    store = lf.AdapterStore(c)
    w = lf.LoraWeight(c)
    torch.nn.init.normal_(w.wa["query"], std=1.0)
    ref = w.wa["query"].clone()
    store.insert("x", w)
    assert torch.equal(store.get("x").wa["query"], ref)
    w.wb["value"].fill_(3.0)  # later edits through the object reach the cache
    slot = store.slot_of("x")
    vi = store.module_index("value")
    assert torch.all(store.cache[slot, vi, 1] == 3.0)


def test_load_from_state_dict_folds_alpha_and_transposes():
    c = cfg(rank=4)
    L, H, R = c.num_layers, c.hidden_size, c.lora_rank
    sd = {}
    g = torch.Generator().manual_seed(3)
    for m in c.target_modules:
        for i in range(L):
            key_a, key_b = lf.peft_key_fn("bert")(i, m)
            sd[key_a] = torch.randn(R, H, generator=g)
            sd[key_b] = torch.randn(H, R, generator=g)
    store = lf.AdapterStore(c)
    store.load_from_state_dict("p", sd, lf.peft_key_fn("bert"), lora_alpha=8)
    w = store.get("p")
    ka, kb = lf.peft_key_fn("bert")(1, "value")
    assert torch.equal(w.wa["value"][1], sd[ka].t())
    assert torch.allclose(w.wb["value"][1], sd[kb].t() * 2.0)
    with pytest.raises(KeyError, match="has no tensor"):
        store.load_from_state_dict("q", {}, lf.peft_key_fn("bert"))


def test_assemblers_match_reference_fixture():
    g = torch.load(GOLD / "assembler.pt", weights_only=False)
    c = cfg()
    store = lf.AdapterStore(c)
    for aid, w in g["weights"].items():
        lw = lf.LoraWeight(c)
        for m in c.target_modules:
            lw.wa[m].copy_(w["wa"][m])
            lw.wb[m].copy_(w["wb"][m])
        store.insert(aid, lw)
    base = BatchAssembler(store, c).assemble_lora(g["ids"])
    for m, layers in g["per_layer_a"].items():
        for layer, ref in enumerate(layers):
            assert torch.equal(torch.cat(base[layer].a[m], 0), ref)
    fast = IndexSelectBatchAssembler(store, c)
    assert fast.batch_index(["adapter_2", "adapter_0", "adapter_2"]).tolist() == g["batch_index"]
    got = fast.assemble_lora(g["ids"])  # CPU store: index_select over the slot views
    for m, (pa, pb) in g["packed"].items():
        assert torch.equal(got[m][0], pa) and torch.equal(got[m][1], pb)
    assert store.memory_bytes() == g["memory_bytes"]


# ------------------------------------------------------------------- heads ---
def test_head_store_validation_and_accounting():
    c = cfg()
    heads = lf.HeadStore(c, capacity_rows=2)
    heads.load("small", torch.randn(3, 32), torch.zeros(3))
    heads.load("big", torch.randn(10, 32), torch.zeros(10))  # forces a regrow
    heads.load("one", torch.randn(32), torch.tensor(0.5))
    assert heads.num_labels("small") == 3 and heads.num_labels("one") == 1
    with pytest.raises(ValueError, match="hidden size"):
        heads.load("bad", torch.randn(3, 33), torch.zeros(3))
    with pytest.raises(ValueError, match="intercept"):
        heads.load("bad", torch.randn(3, 32), torch.zeros(5))
    with pytest.raises(KeyError, match="headless"):
        heads.get("headless")
    table, nl, n_max = heads.head_table(["big", "small", "one"])
    assert nl == [10, 3, 1] and n_max == 10
    coef, bias = heads.packed
    off = table[0].tolist()
    assert torch.equal(coef[off[1] : off[1] + 3], heads.get("small").coef)
    assert heads.memory_bytes() == (3 + 10 + 1) * 33 * 4
    batched = heads.assemble(["small", "big"])
    assert batched.coef.shape == (2, 10, 32) and batched.num_labels == [3, 10]
    assert torch.count_nonzero(batched.coef[0, 3:]) == 0
    heads.evict("small")
    assert "small" not in heads and len(heads) == 2
    heads.load("small2", torch.randn(3, 32), torch.zeros(3))
    assert heads.head_table(["small2"])[0][0].item() == off[1]  # freed rows reused


# ----------------------------------------------------------------- loaders ---
def test_peft_key_fn_naming():
    ka, kb = lf.peft_key_fn("bert")(3, "value")
    assert ka == "base_model.model.encoder.layer.3.attention.self.value.lora_A.weight"
    assert kb == "base_model.model.encoder.layer.3.attention.self.value.lora_B.weight"
    assert "query_proj" in lf.peft_key_fn("deberta-v2")(0, "query")[0]
    assert "attention.output.dense" in lf.peft_key_fn("xlm-roberta")(0, "dense")[0]


@pytest.mark.parametrize("conf,match", [({"r": 8, "lora_alpha": 8, "target_modules": ["query", "value"]}, "rank"),
                                        ({"r": 4, "lora_alpha": 4, "target_modules": ["query", "key"]},
                                         "wrong projections")])
def test_peft_loader_rejects_mismatch(tmp_path, conf, match):
    d = tmp_path / "adapter"
    d.mkdir()
    (d / "adapter_config.json").write_text(json.dumps(conf))
    (d / "adapter_model.bin").write_bytes(b"")
    with pytest.raises(ValueError, match=match):
        lf.load_peft_adapter(lf.AdapterStore(cfg()), "t", str(d))


def _peft_dir(tmp_path, c, rank, alpha, seed):
    """A PEFT adapter directory for the tiny config at ``rank`` (A (r,H), B (H,r) per layer)."""
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for i in range(c.num_layers):
        for m in c.target_modules:
            ka, kb = lf.peft_key_fn("bert")(i, m)
            sd[ka] = torch.randn(rank, c.hidden_size, generator=g)
            sd[kb] = torch.randn(c.hidden_size, rank, generator=g)
    d = tmp_path / f"adapter_r{rank}_{seed}"
    d.mkdir()
    (d / "adapter_config.json").write_text(json.dumps({"r": rank, "lora_alpha": alpha,
                                                        "target_modules": list(c.target_modules)}))
    torch.save(sd, d / "adapter_model.bin")
    return d, sd


def test_mixed_rank_padding_preserves_the_delta(tmp_path):
    """A rank-2 adapter zero-padded into a rank-4 store gives exactly the delta
    (alpha / 2) B A x of the rank-2 adapter, in f32."""
    c = cfg(rank=4)
    store = lf.AdapterStore(c)
    d, sd = _peft_dir(tmp_path, c, rank=2, alpha=6, seed=5)
    with pytest.raises(ValueError, match="rank"):
        lf.load_peft_adapter(store, "low", str(d))  # the reference's default: one rank per pipeline
    lf.load_peft_adapter(store, "low", str(d), pad_rank=True)
    w = store.get("low")
    x = torch.randn(7, c.hidden_size, generator=torch.Generator().manual_seed(1))
    for i in range(c.num_layers):
        for m in c.target_modules:
            ka, kb = lf.peft_key_fn("bert")(i, m)
            want = (x @ sd[ka].T) @ sd[kb].T * (6 / 2)
            got = (x @ w.wa[m][i]) @ w.wb[m][i]
            torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
            assert (w.wa[m][i][:, 2:] == 0).all() and (w.wb[m][i][2:] == 0).all()


@pytest.mark.parametrize("fmt", ["safetensors", "bin"])
def test_registrar_matches_the_reference_fold_bit_for_bit(tmp_path, fmt):
    """A slot staged by the registrar holds the bits of the reference's
    ``LoraWeight.copy_from_tensors``: cast to bf16, transpose, multiply by
    alpha / r in bf16 (``src/latefuse/weights/store.py:51-56``)."""
    from safetensors.torch import save_file

    c = cfg(rank=4, dtype=torch.bfloat16)
    d, sd = _peft_dir(tmp_path, c, rank=4, alpha=12, seed=7)
    if fmt == "safetensors":
        (d / "adapter_model.bin").unlink()
        save_file(sd, str(d / "adapter_model.safetensors"))
    store = lf.AdapterStore(c)
    lf.load_peft_adapter(store, "t", str(d))
    w = store.get("t")
    for m in c.target_modules:
        a = torch.stack([sd[lf.peft_key_fn("bert")(i, m)[0]] for i in range(c.num_layers)])
        b = torch.stack([sd[lf.peft_key_fn("bert")(i, m)[1]] for i in range(c.num_layers)])
        assert torch.equal(w.wa[m], a.to(torch.bfloat16).transpose(1, 2))
        assert torch.equal(w.wb[m], b.to(torch.bfloat16).transpose(1, 2).mul_(12 / 4))


def test_registrar_reports_shapes_and_missing_keys(tmp_path):
    c = cfg(rank=4)
    d, sd = _peft_dir(tmp_path, c, rank=4, alpha=4, seed=8)
    ka, _ = lf.peft_key_fn("bert")(1, "value")
    bad = dict(sd)
    bad[ka] = torch.randn(4, c.hidden_size + 1)
    torch.save(bad, d / "adapter_model.bin")
    with pytest.raises(ValueError, match="expected"):
        lf.load_peft_adapter(lf.AdapterStore(c), "t", str(d))
    del bad[ka]
    torch.save(bad, d / "adapter_model.bin")
    with pytest.raises(KeyError, match="has no tensor"):
        lf.load_peft_adapter(lf.AdapterStore(c), "t", str(d))
    with pytest.raises(FileNotFoundError):
        lf.load_peft_adapter(lf.AdapterStore(c), "t", str(tmp_path / "missing"))


def test_fill_random_refuses_a_resident_id_without_touching_the_store():
    store = lf.AdapterStore(cfg(), capacity=4)
    store.load_synthetic("adapter_1", seed=0)
    before = store.get("adapter_1").wa["query"].clone()
    with pytest.raises(ValueError, match="adapter_1"):
        store.fill_random_(3)
    assert store.adapter_ids() == ["adapter_1"]
    assert torch.equal(store.get("adapter_1").wa["query"], before)
    store.load_synthetic("next", seed=1)  # takes a fresh slot: the resident adapter is untouched
    assert store.slot_of("next") != store.slot_of("adapter_1")
    assert torch.equal(store.get("adapter_1").wa["query"], before)
    ids = store.fill_random_(2, prefix="bulk_")
    assert len({store.slot_of(i) for i in ids + ["adapter_1", "next"]}) == 4


def test_mixed_rank_no_stale_weights_in_a_reused_slot(tmp_path):
    """A padded adapter loaded into the slot a full-rank adapter left behind
    carries none of its columns."""
    c = cfg(rank=4)
    store = lf.AdapterStore(c)
    d4, _ = _peft_dir(tmp_path, c, rank=4, alpha=4, seed=1)
    d2, _ = _peft_dir(tmp_path, c, rank=2, alpha=2, seed=2)
    lf.load_peft_adapter(store, "full", str(d4))
    slot = store.slot_of("full")
    store.evict("full")
    lf.load_peft_adapter(store, "low", str(d2), pad_rank=True)
    assert store.slot_of("low") == slot
    w = store.get("low")
    for m in c.target_modules:
        assert (w.wa[m][:, :, 2:] == 0).all() and (w.wb[m][:, 2:, :] == 0).all()
    d8, _ = _peft_dir(tmp_path, c, rank=8, alpha=8, seed=3)
    with pytest.raises(ValueError, match="rank"):
        lf.load_peft_adapter(store, "high", str(d8), pad_rank=True)  # cannot shrink a rank


# ------------------------------------------------------------------- misc ---
def test_pooling_validation():
    assert lf.validate_pooling("mean") == "mean"
    with pytest.raises(ValueError, match="unknown pooling"):
        lf.validate_pooling("first_token")


def test_every_export_is_importable():
    missing = [n for n in lf.__all__ if not hasattr(lf, n)]
    assert not missing


def test_reference_api_surface_is_mirrored():
    """Every name the reference exports has a counterpart here."""
    reference_all = ["MultiTenantEmbedder", "MultiTenantClassifier", "MultiTenantReranker", "RerankResult",
                     "TaskPipeline", "LoraServingConfig", "load_peft_adapter", "peft_key_fn", "POOLING_STRATEGIES",
                     "AdapterStore", "LoraWeight", "HeadStore", "LRHead", "EncoderWithLora", "HFEncoderWithLora",
                     "BatchAssembler", "IndexSelectBatchAssembler", "BatchedLRWeights", "LayerwiseBatchedWeights",
                     "LoraOps", "LRHeadOps", "__version__"]
    assert not [n for n in reference_all if n not in lf.__all__]
    for cls, methods in {
        lf.TaskPipeline: ["from_pretrained", "register_adapter", "register_synthetic", "evict_adapter", "tenant_ids"],
        lf.MultiTenantEmbedder: ["embed"],
        lf.MultiTenantClassifier: ["logits", "predict_proba", "predict", "encode"],
        lf.MultiTenantReranker: ["score", "rerank"],
        lf.AdapterStore: ["load_from_file", "load_from_state_dict", "load_synthetic", "insert", "get", "evict",
                          "adapter_ids", "memory_bytes", "memory_gb", "config"],
        lf.HeadStore: ["load", "load_from_sklearn", "load_from_file", "assemble", "get", "evict", "tenant_ids",
                       "num_labels", "memory_bytes"],
        lf.IndexSelectBatchAssembler: ["batch_index", "assemble_lora", "to_layerwise"],
        lf.BatchAssembler: ["assemble_lora", "assemble_lr", "assemble"],
        lf.LoraOps: ["shrink", "expand", "output"],
        lf.HFEncoderWithLora: ["encode_pooled", "forward", "close", "from_pretrained_serving"],
        lf.EncoderWithLora: ["encode_pooled", "forward", "from_pretrained_serving", "position_ids"],
    }.items():
        assert not [m for m in methods if not hasattr(cls, m)], cls


def test_unknown_engine_and_assembler_are_rejected():
    class Dummy(torch.nn.Module):
        pass

    with pytest.raises(ValueError, match="unknown engine"):
        lf.TaskPipeline(cfg(), engine="tensorrt", tokenizer=object(), model=Dummy())
    with pytest.raises(ValueError, match="unknown assembler"):
        lf.TaskPipeline(cfg(), assembler="magic", tokenizer=object(), model=Dummy())
    with pytest.raises(ValueError, match="unknown pooling"):
        lf.TaskPipeline(cfg(), pooling="first_token", tokenizer=object(), model=Dummy())


def test_cpu_serving_path_fails_loudly():
    """No CPU fallback: the kernels refuse CPU tensors."""
    from latefuse_b200._native import NativeLibraryError

    with pytest.raises(NativeLibraryError, match="CUDA"):
        lf.pool_tokens(torch.randn(2, 3, 32), None, "cls")


def test_stream_to_host_yields_every_result_in_order_with_bounded_lookahead():
    from latefuse_b200.tasks import stream_to_host

    started = []

    def step(i):
        started.append(i)
        return torch.full((2, 3), float(i))

    seen = []
    for i, host in enumerate(stream_to_host(step, ((i,) for i in range(5)), depth=2)):
        assert torch.equal(host, torch.full((2, 3), float(i)))
        seen.append(i)
        assert len(started) <= i + 2  # never more than depth batches started ahead
    assert seen == list(range(5)) and started == list(range(5))
    assert [h[0, 0].item() for h in stream_to_host(step, [(7,)], depth=1)] == [7.0]
    with pytest.raises(ValueError, match="depth"):
        list(stream_to_host(step, [(0,)], depth=0))


# ------------------------------------------------------- native-rank buckets ---
def test_rank_buckets_keep_each_adapter_at_its_own_rank(tmp_path):
    """PEFT adapters of ranks 2 and 4 in an r_max-8 fleet: each in its own bucket at its
    own rank (the padded store holds both at 8), re-registration at another rank moves
    buckets, and the errors name the tenant or the rank."""
    from latefuse_b200.rank_buckets import RankBucketStore

    c = cfg(rank=8)
    fleet = RankBucketStore(c)
    d2, sd2 = _peft_dir(tmp_path, c, rank=2, alpha=4, seed=1)
    d4, _ = _peft_dir(tmp_path, c, rank=4, alpha=8, seed=2)
    lf.load_peft_adapter(fleet, "two", str(d2))
    lf.load_peft_adapter(fleet, "four", str(d4))
    assert fleet.rank_of("two") == 2 and fleet.rank_of("four") == 4 and fleet.ranks() == [2, 4]
    assert fleet.get("two").wa["query"].shape == (c.num_layers, c.hidden_size, 2)
    padded = lf.AdapterStore(c)
    lf.load_peft_adapter(padded, "two", str(d2), pad_rank=True)
    lf.load_peft_adapter(padded, "four", str(d4), pad_rank=True)
    assert fleet.memory_bytes() * 8 == padded.memory_bytes() * (2 + 4) // 2
    ka, kb = lf.peft_key_fn("bert")(1, "value")
    torch.testing.assert_close(fleet.get("two").wb["value"][1], (sd2[kb] * 2).T.contiguous())
    lf.load_peft_adapter(fleet, "two", str(d4))  # now rank 4: it leaves the rank-2 bucket
    assert fleet.rank_of("two") == 4 and fleet.ranks() == [4] and len(fleet) == 2
    fleet.evict("four")
    assert "four" not in fleet and fleet.adapter_ids() == ["two"]
    with pytest.raises(KeyError, match="nobody"):
        fleet.batch_store(["two", "nobody"])
    d16, _ = _peft_dir(tmp_path, c, rank=16, alpha=16, seed=3)
    with pytest.raises(ValueError, match="rank"):
        lf.load_peft_adapter(fleet, "big", str(d16))
    assert "big" not in fleet


def test_rank_bucket_batch_store_pads_to_r_max_and_reuses_slots_cleanly():
    """The batch staging cache: slot u holds the batch's u-th distinct adapter, its A
    columns and B rows beyond its rank zero, also when the slot held a higher-rank
    adapter in the batch before; the padded slots equal a pad_rank store's."""
    from latefuse_b200.rank_buckets import RankBucketStore

    c = cfg(rank=8)
    fleet = RankBucketStore(c)
    ids = fleet.fill_random_([8, 2, 4, 8, 2], std=0.1, generator=torch.Generator().manual_seed(3))
    assert [fleet.rank_of(a) for a in ids] == [8, 2, 4, 8, 2]
    first = fleet.batch_store([ids[0], ids[3], ids[0]])
    assert first.slots([ids[0], ids[3], ids[0]]) == [0, 1, 0]
    stage = fleet.batch_store([ids[2], ids[1], ids[1], ids[4]])  # slots 0, 1 held rank-8 adapters
    assert stage.slots([ids[1], ids[4], ids[2]]) == [0, 1, 2]  # grouped by rank
    for a in (ids[1], ids[2], ids[4]):
        r, mine, got = fleet.rank_of(a), fleet.get(a), stage.get(a)
        for m in c.target_modules:
            assert torch.equal(got.wa[m][..., :r], mine.wa[m]) and not got.wa[m][..., r:].any()
            assert torch.equal(got.wb[m][:, :r], mine.wb[m]) and not got.wb[m][:, r:].any()
    # the kernels' view of the staging cache is that of a padded store
    fc = stage.factor_cache(1)
    assert fc.rank == 8 and fc.n_slots >= 3
    with pytest.raises(TypeError, match="batch_store"):
        fleet.slots(ids)
