"""The task-level API on the GPU, mirroring the reference's ``tests/test_tasks.py``
(chunking, padding isolation, tenant isolation, pooling, ragged heads, reranking,
assembler/engine equivalence) plus parity with the reference's own outputs on the
same tiny BERT (golden fixture, f32)."""

from __future__ import annotations

import pytest
import torch

import latefuse_b200 as lf
from tests._fixtures import insert_adapters, texts, tiny_bert_dir

pytestmark = pytest.mark.gpu
KW = dict(lora_rank=4, batch_size=8, max_seq_len=16, dtype=torch.float32)


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    return tiny_bert_dir(tmp_path_factory.mktemp("tiny"))


def embedder(tiny, cuda, **kwargs):
    path, g = tiny
    emb = lf.MultiTenantEmbedder.from_pretrained(path, device=cuda, **dict(KW, **kwargs))
    insert_adapters(emb.store, g["adapters"], emb.config)
    return emb


def classifier(tiny, cuda):
    path, g = tiny
    clf = lf.MultiTenantClassifier.from_pretrained(path, device=cuda, **KW)
    insert_adapters(clf.store, g["adapters"], clf.config)
    for t, (c, i) in g["heads"].items():
        clf.heads.load(t, c, i)
    return clf


# --------------------------------------------------------- reference parity ---
@pytest.mark.parametrize("engine", ["hf", "bert"])
def test_embeddings_match_reference(tiny, cuda, engine):
    _, g = tiny
    emb = embedder(tiny, cuda, engine=engine)
    t, ten = g["texts"], g["tenants"]
    torch.testing.assert_close(emb.embed(t, ten).cpu(), g["embed_cls"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(emb.embed(t, ten, pooling="mean").cpu(), g["embed_mean"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(emb.embed(t, ten, normalize=False).cpu(), g["embed_raw"], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(emb.embed(t, ten, pooling="auto").cpu(), g["embed_auto"], atol=1e-5, rtol=1e-5)
    emb.check_device_status()


def test_classifier_and_reranker_match_reference(tiny, cuda):
    path, g = tiny
    clf = classifier(tiny, cuda)
    t, ten = g["clf_texts"], g["clf_tenants"]
    for got, want in zip(clf.logits(t, ten), g["clf_logits"]):
        assert got == pytest.approx(want, abs=1e-4)
    for got, want in zip(clf.predict_proba(t, ten), g["clf_probs"]):
        assert got == pytest.approx(want, abs=1e-5)
    assert clf.predict(t, ten) == g["clf_pred"]
    rr = lf.MultiTenantReranker.from_pretrained(path, device=cuda, **KW)
    insert_adapters(rr.store, {"acme": g["adapters"]["acme"]}, rr.config)
    rr.heads.load("acme", g["rerank_coef"], torch.zeros(1))
    assert rr.score(["tok1 tok2"] * 9, g["rerank_docs"], "acme") == pytest.approx(g["rerank_scores"], abs=1e-4)


# ------------------------------------------------------ reference semantics ---
@pytest.mark.parametrize("n", [1, 7, 8, 9, 20])
def test_embed_accepts_any_length(tiny, cuda, n):
    assert embedder(tiny, cuda).embed(texts(n), "acme").shape == (n, 32)


def test_embed_empty_and_mismatch(tiny, cuda):
    emb = embedder(tiny, cuda)
    assert emb.embed([], []).shape == (0, 32)
    with pytest.raises(ValueError, match="tenant"):
        emb.embed(texts(3), ["acme", "globex"])


def test_padding_does_not_leak(tiny, cuda):
    emb = embedder(tiny, cuda)
    full = emb.embed(texts(16), ["acme", "globex"] * 8)
    short = emb.embed(texts(16)[:3], (["acme", "globex"] * 8)[:3])
    torch.testing.assert_close(short, full[:3], atol=1e-5, rtol=1e-5)
    one = emb.embed([texts(20)[8]], [(["acme", "globex"] * 10)[8]])
    torch.testing.assert_close(one[0], emb.embed(texts(20), ["acme", "globex"] * 10)[8], atol=1e-5, rtol=1e-5)


def test_mixed_batch_matches_per_tenant_batches(tiny, cuda):
    emb = embedder(tiny, cuda)
    t = texts(6)
    mixed = emb.embed(t, ["acme", "globex"] * 3)
    torch.testing.assert_close(mixed[0::2], emb.embed(t[0::2], "acme"), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(mixed[1::2], emb.embed(t[1::2], "globex"), atol=1e-5, rtol=1e-5)
    assert not torch.allclose(emb.embed(t[:1], "acme"), emb.embed(t[:1], "globex"), atol=1e-4)


def test_unknown_tenant_raises(tiny, cuda):
    with pytest.raises(KeyError, match="nobody"):
        embedder(tiny, cuda).embed(texts(1), ["nobody"])


def test_normalisation_and_pooling(tiny, cuda):
    emb = embedder(tiny, cuda)
    norms = emb.embed(texts(5), "acme").norm(dim=-1)
    torch.testing.assert_close(norms, torch.ones_like(norms), atol=1e-5, rtol=1e-5)
    raw = emb.embed(texts(5), "acme", normalize=False).norm(dim=-1)
    assert not torch.allclose(raw, torch.ones_like(raw), atol=1e-3)
    assert not torch.allclose(emb.embed(texts(4), "acme", pooling="cls"), emb.embed(texts(4), "acme", pooling="mean"),
                              atol=1e-3)


def test_ragged_labels_sum_to_one_and_sigmoid(tiny, cuda):
    clf = classifier(tiny, cuda)
    ten = ["acme", "globex", "acme", "globex"]
    probs = clf.predict_proba(texts(4), ten)
    assert [len(p) for p in probs] == [3, 10, 3, 10]
    for row in probs:
        assert sum(row) == pytest.approx(1.0, abs=1e-5)
    preds = clf.predict(texts(4), ten)
    assert all(0 <= p < clf.heads.num_labels(t) for p, t in zip(preds, ten))
    clf.heads.load("acme", torch.randn(1, 32, generator=torch.Generator().manual_seed(3)), torch.zeros(1))
    p1 = clf.predict_proba(texts(2), ["acme", "acme"])
    assert all(len(p) == 1 and 0.0 < p[0] < 1.0 for p in p1)
    assert all(p in (0, 1) for p in clf.predict(texts(2), ["acme", "acme"]))
    clf.register_synthetic("headless", seed=9)
    with pytest.raises(KeyError, match="headless"):
        clf.predict(texts(1), ["headless"])


def test_rerank_orders_descending(tiny, cuda):
    path, g = tiny
    rr = lf.MultiTenantReranker.from_pretrained(path, device=cuda, **KW)
    rr.register_synthetic("acme", seed=5)
    rr.heads.load("acme", torch.randn(1, 32, generator=torch.Generator().manual_seed(4)), torch.zeros(1))
    docs = texts(9)
    ranked = rr.rerank("tok1 tok2", docs, "acme")
    assert [r.score for r in ranked] == sorted((r.score for r in ranked), reverse=True)
    assert sorted(r.index for r in ranked) == list(range(9))
    assert [r.index for r in rr.rerank("tok1 tok2", docs, "acme", top_k=3)] == [r.index for r in ranked[:3]]
    with pytest.raises(ValueError, match="one entry per pair"):
        rr.score(["q", "q"], ["d"], "acme")


def test_assemblers_and_engines_agree(tiny, cuda):
    t, ten = texts(10), ["acme", "globex"] * 5
    a = embedder(tiny, cuda).embed(t, ten)
    b = embedder(tiny, cuda, assembler="index_select").embed(t, ten)
    torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5)
    c = embedder(tiny, cuda, engine="bert").embed(t, ten)
    torch.testing.assert_close(a, c, atol=1e-4, rtol=1e-4)


def test_registering_and_evicting_after_first_use(tiny, cuda):
    emb = embedder(tiny, cuda, assembler="index_select")
    emb.embed(texts(2), "acme")
    emb.register_synthetic("newcomer", seed=42)
    assert emb.embed(texts(2), "newcomer").shape == (2, 32)
    emb.evict_adapter("newcomer")
    with pytest.raises(KeyError, match="newcomer"):
        emb.embed(texts(1), ["newcomer"])


def test_skip_padding_changes_nothing(tiny, cuda):
    path, g = tiny
    a = embedder(tiny, cuda).embed(g["texts"], g["tenants"])
    b = embedder(tiny, cuda, skip_padding=False).embed(g["texts"], g["tenants"])
    torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)
