"""Helpers that rebuild the golden fixtures' tiny models, tokenizers and adapters."""

from __future__ import annotations

import json
from pathlib import Path

import torch

import latefuse_b200 as lf

GOLD = Path(__file__).resolve().parent / "golden"


def load(name: str):
    return torch.load(GOLD / name, weights_only=False)


def tiny_bert_dir(tmp: Path) -> tuple[str, dict]:
    """Save the reference test-suite's tiny BERT (weights + WordPiece vocab) to ``tmp``."""
    from transformers import BertConfig, BertModel

    g = load("tiny_bert_tasks.pt")
    path = tmp / "tiny_bert"
    path.mkdir(parents=True, exist_ok=True)
    model = BertModel(BertConfig(**g["config"])).eval()
    model.load_state_dict(g["state"])
    model.save_pretrained(str(path))
    (path / "vocab.txt").write_text("\n".join(g["vocab"]) + "\n")
    (path / "tokenizer_config.json").write_text(json.dumps({"model_max_length": 512, "tokenizer_class": "BertTokenizer"}))
    return str(path), g


def tiny_xlmr(dtype=torch.float32):
    from transformers import XLMRobertaConfig, XLMRobertaModel

    g = load("tiny_xlmr_dense.pt")
    model = XLMRobertaModel(XLMRobertaConfig(**g["config"])).eval()
    model.load_state_dict(g["state"])
    return model.to(dtype), g


def insert_adapters(store, adapters: dict, config) -> None:
    """Register fixture adapters ``{tenant: {"wa": {m: (L,H,R)}, "wb": ...}}`` in a store."""
    from latefuse_b200 import LoraWeight

    for t, w in adapters.items():
        lw = LoraWeight(config)
        for m in config.target_modules:
            lw.wa[m].copy_(w["wa"][m])
            lw.wb[m].copy_(w["wb"][m])
        store.insert(t, lw)


def texts(n: int) -> list[str]:
    return [f"tok{i % 40} tok{(i * 7) % 40}" for i in range(n)]


def hf_model(kind: str, conf: dict, dev, dtype, seed: int = 0):
    """A HuggingFace encoder with N(0, 0.02) weights, zero biases and unit LayerNorms,
    drawn on ``dev`` from ``seed`` (the models' own initialisation, without the CPU pass)."""
    from transformers import (BertConfig, BertModel, XLMRobertaConfig, XLMRobertaModel, XLMRobertaXLConfig,
                              XLMRobertaXLModel)

    cfg_cls, model_cls = {"bert": (BertConfig, BertModel), "xlmr": (XLMRobertaConfig, XLMRobertaModel),
                          "xlmr-xl": (XLMRobertaXLConfig, XLMRobertaXLModel)}[kind]
    hf = cfg_cls(**conf)
    with torch.device("meta"):
        model = model_cls(hf)
    model = model.to_empty(device=dev).eval()
    g = torch.Generator(device=dev).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "LayerNorm.weight" in name or "layer_norm.weight" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.normal_(0.0, 0.02, generator=g)
        if hf.pad_token_id is not None:
            model.embeddings.word_embeddings.weight[hf.pad_token_id].zero_()
        for name, b in model.named_buffers():
            if name.endswith("position_ids"):
                b.copy_(torch.arange(b.shape[-1], device=dev).expand_as(b))
            else:
                b.zero_()
    return model.to(dtype), hf


def serving_config(hf, dev, dtype, rank, targets, batch, seq):
    return lf.LoraServingConfig(model_name=f"{hf.model_type}-shape (synthetic)", lora_rank=rank, batch_size=batch,
                                max_seq_len=seq, target_modules=list(targets), device=dev, dtype=dtype,
                                hf_config=hf)


def adapters_of(store, tenants) -> dict:
    """The oracle's view of the store's adapters (the slot views themselves)."""
    out = {}
    for t in set(tenants):
        w = store.get(t)
        out[t] = {"wa": dict(w.wa), "wb": dict(w.wb)}
    return out


def row_rel(a, b) -> float:
    a, b = a.float(), b.float()
    return ((a - b).norm(dim=-1) / b.norm(dim=-1).clamp_min(1e-12)).max().item()
