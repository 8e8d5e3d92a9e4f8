"""Generate the golden fixtures in this directory by running the reference itself.

Run here (not on the GPU box), with the reference checkout importable:

    python tests/golden/make_golden.py --reference <reference checkout>/src

Every fixture is produced by the reference's own code on the CPU (LoraOps,
IndexSelectBatchAssembler, BatchAssembler, HeadStore, LRHeadOps, pool_tokens,
AdapterStore.load_synthetic, HFEncoderWithLora / EncoderWithLora and the task
wrappers), on tiny seeded models, so the fixtures stay small.  The tests check
the oracle and the GPU path against them; nothing at test time imports the
reference.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _save(name: str, obj) -> None:
    torch.save(obj, HERE / name)
    print(f"wrote {name} ({(HERE / name).stat().st_size} bytes)")


def _bert_dir(tmp: Path, **cfg) -> str:
    from transformers import BertConfig

    path = tmp / f"bert_{cfg['hidden_size']}_{cfg['num_hidden_layers']}"
    path.mkdir(parents=True, exist_ok=True)
    BertConfig(**cfg).save_pretrained(str(path))
    return str(path)


TINY = dict(vocab_size=100, hidden_size=32, num_hidden_layers=2, num_attention_heads=4, intermediate_size=64,
            max_position_embeddings=64, pad_token_id=0)


def gen_lora_ops(tmp: Path) -> None:
    from latefuse.config import LoraServingConfig
    from latefuse.ops.lora import LoraOps

    model = _bert_dir(tmp, **dict(TINY, hidden_size=64, num_attention_heads=4, intermediate_size=128))
    out = {}
    for dtype in (torch.float32, torch.bfloat16):
        cfg = LoraServingConfig(model_name=model, lora_rank=8, batch_size=3, max_seq_len=8,
                                target_modules=["query", "value"], device=torch.device("cpu"), dtype=dtype)
        g = torch.Generator().manual_seed(1234)
        B, S, H, R = 3, 8, 64, 8
        x = torch.randn(B, S, H, generator=g).to(dtype)
        a = (torch.randn(B, H, R, generator=g) * 0.05).to(dtype)
        b = (torch.randn(B, R, H, generator=g) * 0.05).to(dtype)
        base = torch.randn(B, S, H, generator=g).to(dtype)
        ops = LoraOps(cfg)
        ops.shrink(x, a)
        ops.expand(b)
        out[str(dtype)] = dict(x=x, a=a, b=b, base=base, out_A=ops._out_A.clone(), out_B=ops.output.clone(),
                               hooked=base + ops.output)
    _save("lora_ops.pt", out)


def gen_assembler(tmp: Path) -> None:
    from latefuse.config import LoraServingConfig
    from latefuse.weights.batch import BatchAssembler, IndexSelectBatchAssembler
    from latefuse.weights.store import AdapterStore

    cfg = LoraServingConfig(model_name=_bert_dir(tmp, **TINY), lora_rank=4, batch_size=4, max_seq_len=16,
                            target_modules=["query", "value"], device=torch.device("cpu"), dtype=torch.float32)
    store = AdapterStore(cfg)
    for i in range(6):
        store.load_synthetic(f"adapter_{i}", seed=100 + i)
        torch.nn.init.normal_(store.get(f"adapter_{i}").wb["query"], std=0.02)
    ids = ["adapter_3", "adapter_0", "adapter_3", "adapter_5"]
    base = BatchAssembler(store, cfg).assemble_lora(ids)
    fast = IndexSelectBatchAssembler(store, cfg)
    packed = fast.assemble_lora(ids)
    weights = {aid: {"wa": {m: w.wa[m].clone() for m in w.wa}, "wb": {m: w.wb[m].clone() for m in w.wb}}
               for aid in store.adapter_ids() for w in [store.get(aid)]}
    per_layer = {m: [torch.cat(base[l].a[m], 0) for l in range(cfg.num_layers)] for m in cfg.target_modules}
    _save("assembler.pt", dict(ids=ids, weights=weights, packed=packed, per_layer_a=per_layer,
                               batch_index=fast.batch_index(["adapter_2", "adapter_0", "adapter_2"]).tolist(),
                               memory_bytes=store.memory_bytes()))


def gen_synthetic_rng(tmp: Path) -> None:
    from latefuse.config import LoraServingConfig
    from latefuse.weights.store import AdapterStore

    cfg = LoraServingConfig(model_name=_bert_dir(tmp, **TINY), lora_rank=4, batch_size=4, max_seq_len=16,
                            target_modules=["query", "value"], device=torch.device("cpu"), dtype=torch.float32)
    store = AdapterStore(cfg)
    store.load_synthetic("a", seed=7)
    w = store.get("a")
    _save("synthetic_rng.pt", dict(seed=7, wa={m: w.wa[m].clone() for m in w.wa},
                                   wb={m: w.wb[m].clone() for m in w.wb}))


def gen_heads_and_pooling(tmp: Path) -> None:
    from latefuse.config import LoraServingConfig
    from latefuse.ops.head import LRHeadOps
    from latefuse.ops.pooling import pool_tokens
    from latefuse.tasks.classification import _sigmoid, _softmax
    from latefuse.tasks.heads import HeadStore

    out = {}
    for dtype in (torch.float32, torch.bfloat16):
        cfg = LoraServingConfig(model_name=_bert_dir(tmp, **TINY), lora_rank=4, batch_size=4, max_seq_len=16,
                                target_modules=["query", "value"], device=torch.device("cpu"), dtype=dtype)
        g = torch.Generator().manual_seed(99)
        H = 32
        heads = HeadStore(cfg)
        spec = {"small": 3, "big": 10, "one": 1}
        raw = {}
        for t, n in spec.items():
            coef = torch.randn(n, H, generator=g) * 0.5
            icpt = torch.randn(n, generator=g) * 0.1
            heads.load(t, coef, icpt)
            raw[t] = (coef, icpt)
        tenants = ["small", "big", "one", "small", "big"]
        pooled = torch.randn(len(tenants), H, generator=g).to(dtype)
        batched = heads.assemble(tenants)
        o = torch.zeros(len(tenants), 1, batched.coef.shape[1], dtype=dtype)
        LRHeadOps.predict_proba(pooled.unsqueeze(1), batched.coef, batched.intercept, o)
        scores = o[:, 0]
        logits = [scores[i, :n].tolist() for i, n in enumerate(batched.num_labels)]
        probs = [_sigmoid(r) if len(r) == 1 else _softmax(r) for r in logits]
        hidden = torch.randn(3, 8, H, generator=g).to(dtype)
        mask = torch.tensor([[1] * 8, [1] * 5 + [0] * 3, [1] * 2 + [0] * 6])
        out[str(dtype)] = dict(raw=raw, tenants=tenants, pooled=pooled, padded_logits=o.clone(), logits=logits,
                               probs=probs, num_labels=batched.num_labels, hidden=hidden, mask=mask,
                               cls=pool_tokens(hidden, mask, "cls").clone(), mean=pool_tokens(hidden, mask, "mean"),
                               mean_nomask=pool_tokens(hidden, None, "mean"),
                               normalized=torch.nn.functional.normalize(pooled, p=2, dim=-1))
    _save("heads_pooling.pt", out)


def _tiny_tokenizer_files(path: Path) -> list[str]:
    vocab = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] + [f"tok{i}" for i in range(TINY["vocab_size"] - 5)]
    (path / "vocab.txt").write_text("\n".join(vocab) + "\n")
    (path / "tokenizer_config.json").write_text(json.dumps({"model_max_length": 512, "tokenizer_class": "BertTokenizer"}))
    return vocab


def _texts(n: int) -> list[str]:
    return [f"tok{i % 40} tok{(i * 7) % 40}" for i in range(n)]


def gen_tiny_bert_tasks(tmp: Path) -> None:
    """The reference's task wrappers on the tiny BERT of its own test-suite."""
    from transformers import BertConfig, BertModel

    from latefuse import MultiTenantClassifier, MultiTenantEmbedder, MultiTenantReranker

    path = tmp / "tiny_model"
    torch.manual_seed(0)
    BertModel(BertConfig(**TINY)).eval().save_pretrained(str(path))
    vocab = _tiny_tokenizer_files(path)
    state = {k: v.clone() for k, v in BertModel.from_pretrained(str(path)).state_dict().items()}
    kw = dict(lora_rank=4, batch_size=8, max_seq_len=16, device="cpu", dtype=torch.float32)

    def embedder(engine):
        emb = MultiTenantEmbedder.from_pretrained(str(path), engine=engine, **kw)
        for i, tenant in enumerate(("acme", "globex")):
            emb.register_synthetic(tenant, seed=100 + i)
            w = emb.store.get(tenant)
            torch.manual_seed(200 + i)
            for module in emb.config.target_modules:
                torch.nn.init.normal_(w.wb[module], std=0.05)
        emb._invalidate_assembler()
        return emb

    emb = embedder("hf")
    adapters = {t: {"wa": {m: w.wa[m].clone() for m in w.wa}, "wb": {m: w.wb[m].clone() for m in w.wb}}
                for t in ("acme", "globex") for w in [emb.store.get(t)]}
    texts, tenants = _texts(10), ["acme", "globex"] * 5
    res = dict(state=state, vocab=vocab, config=TINY, adapters=adapters, texts=texts, tenants=tenants,
               embed_cls=emb.embed(texts, tenants), embed_mean=emb.embed(texts, tenants, pooling="mean"),
               embed_raw=emb.embed(texts, tenants, normalize=False), embed_auto=emb.embed(texts, tenants, pooling="auto"))
    bert = embedder("bert")
    res["embed_cls_bert_engine"] = bert.embed(texts, tenants, pooling="cls")

    clf = MultiTenantClassifier.from_pretrained(str(path), **kw)
    for i, tenant in enumerate(("acme", "globex")):
        clf.store.insert(tenant, emb.store.get(tenant))
    g = torch.Generator().manual_seed(11)
    heads = {"acme": (torch.randn(3, 32, generator=g), torch.randn(3, generator=g) * 0.1),
             "globex": (torch.randn(10, 32, generator=g), torch.randn(10, generator=g) * 0.1)}
    for t, (c, i) in heads.items():
        clf.heads.load(t, c, i)
    c_texts, c_tenants = _texts(6), ["acme", "globex", "acme", "globex", "globex", "acme"]
    res.update(heads=heads, clf_texts=c_texts, clf_tenants=c_tenants, clf_logits=clf.logits(c_texts, c_tenants),
               clf_probs=clf.predict_proba(c_texts, c_tenants), clf_pred=clf.predict(c_texts, c_tenants))

    rr = MultiTenantReranker.from_pretrained(str(path), **kw)
    rr.store.insert("acme", emb.store.get("acme"))
    rcoef = torch.randn(1, 32, generator=g)
    rr.heads.load("acme", rcoef, torch.zeros(1))
    docs = _texts(9)
    res.update(rerank_coef=rcoef, rerank_docs=docs, rerank_scores=rr.score(["tok1 tok2"] * 9, docs, "acme"))
    _save("tiny_bert_tasks.pt", res)


def gen_tiny_xlmr_dense(tmp: Path) -> None:
    """The reference hf engine on a tiny XLM-R with LoRA on query/key/value and the
    attention-output dense projection (mapped onto attention.output.dense)."""
    from transformers import XLMRobertaConfig, XLMRobertaModel

    import latefuse.model.hf_wrapper as hfw
    from latefuse.config import LoraServingConfig
    from latefuse.model.hf_wrapper import HFEncoderWithLora
    from latefuse.weights.batch import IndexSelectBatchAssembler
    from latefuse.weights.store import AdapterStore

    hfw._TARGET_SUFFIXES["default"]["dense"] = "attention.output.dense"
    conf = dict(vocab_size=120, hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=128,
                max_position_embeddings=80, pad_token_id=1, type_vocab_size=1, layer_norm_eps=1e-5)
    path = tmp / "tiny_xlmr"
    torch.manual_seed(0)
    base = XLMRobertaModel(XLMRobertaConfig(**conf)).eval()
    base.save_pretrained(str(path))
    targets = ["query", "key", "value", "dense"]
    cfg = LoraServingConfig(model_name=str(path), lora_rank=8, batch_size=3, max_seq_len=20, target_modules=targets,
                            device=torch.device("cpu"), dtype=torch.float32)
    model = HFEncoderWithLora(base, cfg).eval()
    store = AdapterStore(cfg)
    for i in range(4):
        store.load_synthetic(f"t{i}", seed=i)
        torch.manual_seed(50 + i)
        for m in targets:
            torch.nn.init.normal_(store.get(f"t{i}").wb[m], std=0.05)
    tenants = ["t2", "t0", "t2"]
    g = torch.Generator().manual_seed(5)
    lengths = [20, 13, 6]
    ids = torch.randint(5, 120, (3, 20), generator=g)
    mask = (torch.arange(20).unsqueeze(0) < torch.tensor(lengths).unsqueeze(1)).long()
    ids = torch.where(mask.bool(), ids, torch.full_like(ids, 1))
    ids[:, 0] = 0
    asm = IndexSelectBatchAssembler(store, cfg)
    with torch.no_grad():
        pooled_cls = model.encode_pooled(ids, mask, asm.to_layerwise(tenants), pooling="cls")
        pooled_mean = model.encode_pooled(ids, mask, asm.to_layerwise(tenants), pooling="mean")
        base_cls = model.encode_pooled(ids, mask, asm.to_layerwise(tenants), apply_lora=False, pooling="cls")
    adapters = {t: {"wa": {m: store.get(t).wa[m].clone() for m in targets},
                    "wb": {m: store.get(t).wb[m].clone() for m in targets}} for t in store.adapter_ids()}
    _save("tiny_xlmr_dense.pt", dict(config=conf, state={k: v.clone() for k, v in base.state_dict().items()},
                                     targets=targets, adapters=adapters, tenants=tenants, ids=ids, mask=mask,
                                     pooled_cls=pooled_cls, pooled_mean=pooled_mean, base_cls=base_cls))


def gen_chunking() -> None:
    from latefuse.tasks.batching import chunk_and_pad

    cases = {}
    for n, bs in [(5, 3), (4, 2), (0, 4), (1, 8), (9, 8), (20, 8)]:
        cases[f"{n}_{bs}"] = [[c, k] for c, k in chunk_and_pad(list(range(n)), bs)]
    (HERE / "chunking.json").write_text(json.dumps(cases, indent=0))
    print("wrote chunking.json")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LATEFUSE_REFERENCE_SRC"),
                    help="the reference checkout's src/ directory (or set LATEFUSE_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <checkout>/src or set LATEFUSE_REFERENCE_SRC")
    sys.path.insert(0, args.reference)
    os.environ.setdefault("HF_HUB_OFFLINE", "1")
    torch.set_num_threads(4)
    with tempfile.TemporaryDirectory() as d:
        tmp = Path(d)
        gen_lora_ops(tmp)
        gen_assembler(tmp)
        gen_synthetic_rng(tmp)
        gen_heads_and_pooling(tmp)
        gen_tiny_bert_tasks(tmp)
        gen_tiny_xlmr_dense(tmp)
        gen_chunking()


if __name__ == "__main__":
    main()
