"""Pin the oracle against golden vectors produced by the reference itself.

``tests/golden/make_golden.py`` ran the reference's own code (LoraOps,
assemblers, AdapterStore, HeadStore, LRHeadOps, pool_tokens, the "hf" and
"bert" engines and the task wrappers) on seeded inputs; these tests check the
oracle's restatement reproduces every fixture.  CPU only.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from oracle import head as oh
from oracle import lora as ol
from oracle import tasks as ot
from oracle.encoder import HookedEncoder, build_model

GOLD = Path(__file__).resolve().parent / "golden"


def load(name):
    return torch.load(GOLD / name, weights_only=False)


# ---------------------------------------------------------------- LoRA op ---
def test_lora_ops_fp32_matches_reference():
    g = load("lora_ops.pt")["torch.float32"]
    d = ol.lora_delta(g["x"], g["a"], g["b"])
    torch.testing.assert_close(d, g["out_B"], atol=1e-5, rtol=0)
    torch.testing.assert_close(torch.bmm(g["x"], g["a"]), g["out_A"], atol=1e-5, rtol=0)
    torch.testing.assert_close(ol.hook_output(g["base"], g["x"], g["a"], g["b"]), g["hooked"], atol=1e-5, rtol=0)
    torch.testing.assert_close(ol.lora_delta_loop(g["x"], g["a"], g["b"]), g["out_B"], atol=1e-5, rtol=0)


def test_lora_ops_bf16_matches_reference():
    g = load("lora_ops.pt")["torch.bfloat16"]
    d = ol.lora_delta(g["x"], g["a"], g["b"]).float()
    ref = g["out_B"].float()
    assert ((d - ref).norm() / ref.norm()).item() < 2e-2
    u = torch.bmm(g["x"].float(), g["a"].float()).to(torch.bfloat16).float()
    assert ((u - g["out_A"].float()).abs().max() <= 2e-2 * g["out_A"].float().abs().max()).item()


def test_segmented_apply_equals_batched_form():
    g = load("lora_ops.pt")["torch.float32"]
    x, a, b, base = g["x"], g["a"], g["b"], g["base"]
    B, S, H = x.shape
    segs = [(i * S, S, i) for i in range(B)]
    out = ol.segmented_apply(x.reshape(-1, H), base.reshape(-1, H), lambda s, m: a[s], lambda s, m: b[s], segs)
    torch.testing.assert_close(out.view(B, S, H), g["hooked"], atol=1e-5, rtol=0)


# ----------------------------------------------------------- assemblers ---
def test_gather_is_bit_exact_against_reference():
    g = load("assembler.pt")
    order = list(g["weights"])
    row_of = {aid: i for i, aid in enumerate(order)}
    for m, (pa, pb) in g["packed"].items():
        stacked_a = torch.stack([g["weights"][aid]["wa"][m] for aid in order])
        stacked_b = torch.stack([g["weights"][aid]["wb"][m] for aid in order])
        assert torch.equal(ol.index_select_gather(stacked_a, row_of, g["ids"]), pa)
        assert torch.equal(ol.index_select_gather(stacked_b, row_of, g["ids"]), pb)
    for m, layers in g["per_layer_a"].items():
        for layer, ref in enumerate(layers):
            got = ol.cpu_assemble(lambda aid: g["weights"][aid]["wa"][m], g["ids"], layer)
            assert torch.equal(got, ref)
    assert [row_of[a] for a in ["adapter_2", "adapter_0", "adapter_2"]] == g["batch_index"] == [2, 0, 2]


def test_synthetic_draws_match_reference():
    g = load("synthetic_rng.pt")
    torch.manual_seed(g["seed"])
    for m, ref in g["wa"].items():
        w = torch.zeros_like(ref)
        torch.nn.init.normal_(w, std=0.02)
        assert torch.equal(w, ref)
    for ref in g["wb"].values():
        assert torch.count_nonzero(ref) == 0


# --------------------------------------------------------- heads/pooling ---
@pytest.mark.parametrize("dtype", ["torch.float32", "torch.bfloat16"])
def test_heads_and_pooling_match_reference(dtype):
    g = load("heads_pooling.pt")[dtype]
    dt = getattr(torch, dtype.split(".")[1])
    coef, icpt, nl = oh.assemble_heads(g["raw"], g["tenants"], 32, dt)
    assert nl == g["num_labels"]
    logits = oh.head_logits(g["pooled"], coef, icpt)
    tol = 1e-5 if dt == torch.float32 else 2e-2
    ref = g["padded_logits"][:, 0].float()
    assert (logits.float() - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    rag = oh.ragged(logits, nl)
    assert [len(r) for r in rag] == [len(r) for r in g["logits"]]
    for got, want in zip(oh.probabilities(rag), g["probs"]):
        assert got == pytest.approx(want, abs=tol)
    torch.testing.assert_close(oh.pool_tokens(g["hidden"], g["mask"], "cls"), g["cls"], atol=0, rtol=0)
    torch.testing.assert_close(oh.pool_tokens(g["hidden"], g["mask"], "mean").float(), g["mean"].float(),
                               atol=tol, rtol=0)
    torch.testing.assert_close(oh.pool_tokens(g["hidden"], None, "mean").float(), g["mean_nomask"].float(),
                               atol=tol, rtol=0)
    torch.testing.assert_close(oh.normalize(g["pooled"]).float(), g["normalized"].float(), atol=tol, rtol=0)


def test_chunking_matches_reference():
    cases = json.loads((GOLD / "chunking.json").read_text())
    for key, want in cases.items():
        n, bs = map(int, key.split("_"))
        assert [[c, k] for c, k in ot.chunk_and_pad(list(range(n)), bs)] == want
    with pytest.raises(ValueError, match="must be positive"):
        list(ot.chunk_and_pad([1], 0))


# -------------------------------------------------------------- encoders ---
def tiny_bert(g, tmp_path):
    from transformers import BertConfig, BertModel, BertTokenizer

    (tmp_path / "vocab.txt").write_text("\n".join(g["vocab"]) + "\n")
    tok = BertTokenizer(str(tmp_path / "vocab.txt"))
    model = build_model(BertConfig, BertModel, g["config"], g["state"])
    return model, tok


def test_tiny_bert_embeddings_match_reference(tmp_path):
    g = load("tiny_bert_tasks.pt")
    model, tok = tiny_bert(g, tmp_path)
    enc = HookedEncoder(model, g["adapters"], ["query", "value"])
    kw = dict(batch_size=8, max_seq_len=16)
    for pooling, key, norm in [("cls", "embed_cls", True), ("mean", "embed_mean", True), ("cls", "embed_raw", False),
                               ("auto", "embed_auto", True)]:
        got = ot.embed(enc, tok, g["texts"], g["tenants"], pooling=pooling, do_normalize=norm, **kw)
        torch.testing.assert_close(got, g[key], atol=1e-5, rtol=1e-5)
    # the reference's two engines agree (the property the oracle inherits)
    torch.testing.assert_close(g["embed_cls_bert_engine"], g["embed_cls"], atol=1e-4, rtol=1e-4)


def test_tiny_bert_classifier_and_reranker_match_reference(tmp_path):
    g = load("tiny_bert_tasks.pt")
    model, tok = tiny_bert(g, tmp_path)
    enc = HookedEncoder(model, g["adapters"], ["query", "value"])
    pooled = ot.embed(enc, tok, g["clf_texts"], g["clf_tenants"], pooling="auto", do_normalize=False,
                      batch_size=8, max_seq_len=16)
    coef, icpt, nl = oh.assemble_heads(g["heads"], g["clf_tenants"], 32, torch.float32)
    logits = oh.ragged(oh.head_logits(pooled, coef, icpt), nl)
    for got, want in zip(logits, g["clf_logits"]):
        assert got == pytest.approx(want, abs=1e-4)
    for got, want in zip(oh.probabilities(logits), g["clf_probs"]):
        assert got == pytest.approx(want, abs=1e-5)
    assert oh.predictions(logits) == g["clf_pred"]
    rp = ot.embed(enc, tok, ["tok1 tok2"] * 9, ["acme"] * 9, text_pairs=g["rerank_docs"], pooling="auto",
                  do_normalize=False, batch_size=8, max_seq_len=16)
    scores = (rp @ g["rerank_coef"][0]).tolist()
    assert scores == pytest.approx(g["rerank_scores"], abs=1e-4)


def test_tiny_xlmr_dense_targets_match_reference():
    from transformers import XLMRobertaConfig, XLMRobertaModel

    g = load("tiny_xlmr_dense.pt")
    model = build_model(XLMRobertaConfig, XLMRobertaModel, g["config"], g["state"])
    enc = HookedEncoder(model, g["adapters"], g["targets"])
    torch.testing.assert_close(enc.encode_pooled(g["ids"], g["mask"], g["tenants"], "cls"), g["pooled_cls"],
                               atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(enc.encode_pooled(g["ids"], g["mask"], g["tenants"], "mean"), g["pooled_mean"],
                               atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(enc.encode_pooled(g["ids"], g["mask"], g["tenants"], "cls", apply_lora=False),
                               g["base_cls"], atol=1e-5, rtol=1e-5)
