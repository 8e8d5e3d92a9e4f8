"""Helpers that rebuild the golden fixtures' tiny models, tokenizers and adapters."""

from __future__ import annotations

import json
from pathlib import Path

import torch

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
