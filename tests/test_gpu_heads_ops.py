"""GPU parity of the head kernel (pool / normalise / gather-GEMV / softmax), the
slot gather, and the reference-shaped ``LoraOps`` / ``LRHeadOps`` APIs, against
the reference's golden fixtures and the oracle."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch
from transformers import BertConfig

import latefuse_b200 as lf
from latefuse_b200.head import head_forward, l2_normalize
from oracle import head as oh

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
TINY = dict(vocab_size=100, hidden_size=32, num_hidden_layers=2, num_attention_heads=4, intermediate_size=64,
            max_position_embeddings=64, pad_token_id=0)


def load(name):
    return torch.load(GOLD / name, weights_only=False)


def cfg(dev, dtype=torch.float32, rank=4, H=32, B=4, S=16):
    return lf.LoraServingConfig(model_name="tiny", lora_rank=rank, batch_size=B, max_seq_len=S,
                                target_modules=["query", "value"], device=dev, dtype=dtype,
                                hf_config=BertConfig(**dict(TINY, hidden_size=H)))


@pytest.mark.parametrize("dtype", ["torch.float32", "torch.bfloat16"])
def test_heads_kernel_matches_reference(cuda, dtype):
    g = load("heads_pooling.pt")[dtype]
    dt = getattr(torch, dtype.split(".")[1])
    heads = lf.HeadStore(cfg(cuda, dt))
    for t, (c, i) in g["raw"].items():
        heads.load(t, c, i)
    table, nl, n_max = heads.head_table(g["tenants"])
    coef, bias = heads.packed
    pooled = g["pooled"].to(cuda)
    logits = torch.empty(len(nl), n_max, dtype=dt, device=cuda)
    probs = torch.empty(len(nl), n_max, dtype=torch.float32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    head_forward(pooled, pooling="none", coef=coef, bias=bias, head_table=table, n_max=n_max, logits_out=logits,
                 probs_out=probs, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    tol = 1e-5 if dt == torch.float32 else 2e-2
    ref = g["padded_logits"][:, 0].float()
    assert (logits.cpu().float() - ref).abs().max().item() <= tol * max(1.0, ref.abs().max().item())
    got_probs = probs.cpu()
    for i, (want, n) in enumerate(zip(g["probs"], nl)):
        assert got_probs[i, :n].tolist() == pytest.approx(want, abs=1e-5 if dt == torch.float32 else 2e-2)
        assert torch.count_nonzero(got_probs[i, n:]) == 0  # padded lanes are not classes
        assert torch.count_nonzero(logits[i, n:]) == 0
    # the oracle on the kernel's own logits gives the kernel's probabilities
    rag = [logits.cpu().float()[i, :n].tolist() for i, n in enumerate(nl)]
    for got, want in zip(oh.probabilities(rag), got_probs.tolist()):
        assert got == pytest.approx(want[: len(got)], abs=1e-6)


@pytest.mark.parametrize("dtype", ["torch.float32", "torch.bfloat16"])
def test_pooling_and_normalize_match_reference(cuda, dtype):
    g = load("heads_pooling.pt")[dtype]
    tol = 1e-6 if dtype == "torch.float32" else 1e-2
    hidden, mask = g["hidden"].to(cuda), g["mask"].to(cuda)
    assert torch.equal(lf.pool_tokens(hidden, mask, "cls").cpu(), g["cls"])
    torch.testing.assert_close(lf.pool_tokens(hidden, mask, "mean").cpu().float(), g["mean"].float(), atol=tol, rtol=0)
    torch.testing.assert_close(lf.pool_tokens(hidden, None, "mean").cpu().float(), g["mean_nomask"].float(),
                               atol=tol, rtol=0)
    torch.testing.assert_close(l2_normalize(g["pooled"].to(cuda)).cpu().float(), g["normalized"].float(),
                               atol=tol, rtol=0)


def test_lr_head_ops_matches_reference(cuda):
    g = load("heads_pooling.pt")["torch.float32"]
    coef, icpt, _ = oh.assemble_heads(g["raw"], g["tenants"], 32, torch.float32)
    out = torch.zeros(len(g["tenants"]), 1, coef.shape[1], device=cuda)
    lf.LRHeadOps.predict_proba(g["pooled"].to(cuda).unsqueeze(1), coef.to(cuda), icpt.to(cuda), out)
    torch.testing.assert_close(out.cpu(), g["padded_logits"], atol=1e-5, rtol=0)


def test_bad_head_range_sets_status(cuda):
    heads = lf.HeadStore(cfg(cuda))
    heads.load("a", torch.randn(3, 32), torch.zeros(3))
    coef, bias = heads.packed
    rows = coef.shape[0]
    table = torch.tensor([[0, rows - 1], [3, 3]], dtype=torch.int32, device=cuda)  # row 1 runs past the cache
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    logits = torch.empty(2, 3, device=cuda)
    head_forward(torch.randn(2, 32, device=cuda), pooling="none", coef=coef, bias=bias, head_table=table, n_max=3,
                 logits_out=logits, status=status)
    torch.cuda.synchronize()
    assert status.item() & 8
    assert torch.count_nonzero(logits[1]) == 0


def test_slot_gather_is_bit_exact(cuda):
    g = load("assembler.pt")
    c = cfg(cuda)
    store = lf.AdapterStore(c)
    for aid, w in g["weights"].items():
        lw = lf.LoraWeight(c)
        for m in c.target_modules:
            lw.wa[m].copy_(w["wa"][m])
            lw.wb[m].copy_(w["wb"][m])
        store.insert(aid, lw)
    fast = lf.IndexSelectBatchAssembler(store, c)
    got = fast.assemble_lora(g["ids"])  # native gather kernel
    for m, (pa, pb) in g["packed"].items():
        assert torch.equal(got[m][0].cpu(), pa) and torch.equal(got[m][1].cpu(), pb)
    assert fast.batch_index(["adapter_2", "adapter_0", "adapter_2"]).tolist() == g["batch_index"]
    layer = fast.to_layerwise(g["ids"])
    assert torch.equal(layer[1].a["query"][0].cpu(), g["per_layer_a"]["query"][1])


@pytest.mark.parametrize("dtype", ["torch.float32", "torch.bfloat16"])
def test_lora_ops_api_matches_reference(cuda, dtype):
    g = load("lora_ops.pt")[dtype]
    dt = getattr(torch, dtype.split(".")[1])
    c = lf.LoraServingConfig(model_name="tiny", lora_rank=8, batch_size=3, max_seq_len=8,
                             target_modules=["query", "value"], device=cuda, dtype=dt,
                             hf_config=BertConfig(**dict(TINY, hidden_size=64)))
    ops = lf.LoraOps(c)
    ops.shrink(g["x"].to(cuda), g["a"].to(cuda))
    ops.expand(g["b"].to(cuda))
    torch.cuda.synchronize()
    if dt == torch.float32:
        torch.testing.assert_close(ops._out_A.cpu(), g["out_A"], atol=1e-5, rtol=0)
        torch.testing.assert_close(ops.output.cpu(), g["out_B"], atol=1e-5, rtol=0)
    else:
        for got, ref in ((ops._out_A.cpu().float(), g["out_A"].float()), (ops.output.cpu().float(), g["out_B"].float())):
            assert ((got - ref).norm() / ref.norm()).item() < 2e-2
    with pytest.raises(AssertionError, match="buffer shape"):
        ops.shrink(torch.zeros(2, 8, 64, device=cuda, dtype=dt), g["a"].to(cuda))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("pooler", [True, False])
def test_head_rows_gather_pooler_head_softmax(cuda, dtype, pooler):
    """``lf_head_forward_rows`` on packed rows against the reference's steps done
    one by one with torch: gather each row's CLS token, the HF pooler
    ``tanh(F.linear(cls, W, b))`` (each result in the dtype), then the oracle's
    zero-padded head bmm + add and the host softmax / sigmoid.  37 rows span three
    row blocks of the pooler; H = 1024 spans sixteen column blocks."""
    from latefuse_b200.head import head_forward_rows

    g = torch.Generator().manual_seed(0)
    T, B, H = 900, 37, 1024
    hidden = torch.randn(T, H, generator=g).to(dtype).to(cuda)
    rows = torch.randperm(T, generator=g)[:B].to(torch.int32)
    W = (torch.randn(H, H, generator=g) * H ** -0.5).to(dtype).to(cuda)
    b = (torch.randn(H, generator=g) * 0.1).to(dtype).to(cuda)
    heads = lf.HeadStore(cfg(cuda, dtype, H=H))
    raw = {}
    for i in range(9):
        n = 1 if i == 4 else int(torch.randint(2, 21, (1,), generator=g))
        raw[f"t{i}"] = (torch.randn(n, H, generator=g) * 0.05, torch.randn(n, generator=g) * 0.1)
        heads.load(f"t{i}", *raw[f"t{i}"])
    tenants = [f"t{int(i)}" for i in torch.randint(0, 9, (B,), generator=g)]
    table, nl, n_max = heads.head_table(tenants)
    coef, bias = heads.packed
    pooled = torch.empty(B, H, dtype=dtype, device=cuda)
    logits = torch.empty(B, n_max, dtype=dtype, device=cuda)
    probs = torch.empty(B, n_max, dtype=torch.float32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    head_forward_rows(hidden, rows.to(cuda), pooler_w=W if pooler else None, pooler_b=b if pooler else None,
                      pooled_out=pooled, coef=coef, bias=bias, head_table=table, n_max=n_max, logits_out=logits,
                      probs_out=probs, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    cls = hidden.index_select(0, rows.to(cuda).long())
    want_pooled = torch.tanh(torch.nn.functional.linear(cls, W, b)) if pooler else cls
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    if pooler:
        assert (pooled.float() - want_pooled.float()).abs().max().item() <= tol
    else:
        assert torch.equal(pooled, want_pooled)  # a gather is exact
    c_ref, i_ref, nl_ref = oh.assemble_heads({t: (c.to(dtype), i.to(dtype)) for t, (c, i) in raw.items()}, tenants,
                                             H, dtype)
    assert nl == nl_ref
    ref_logits = oh.head_logits(want_pooled.cpu(), c_ref, i_ref).float()
    scale = max(1.0, ref_logits.abs().max().item())
    for i, n in enumerate(nl):
        assert (logits[i, :n].float().cpu() - ref_logits[i, :n]).abs().max().item() <= tol * scale
        assert torch.count_nonzero(logits[i, n:]) == 0 and torch.count_nonzero(probs[i, n:]) == 0
    ref_probs = oh.probabilities(oh.ragged(ref_logits, nl))
    for i, n in enumerate(nl):
        assert probs[i, :n].cpu().tolist() == pytest.approx(ref_probs[i], abs=1e-5 if dtype == torch.float32
                                                            else 2e-2)
