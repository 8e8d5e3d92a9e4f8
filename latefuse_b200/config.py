"""Serving configuration (mirror of ``src/latefuse/config.py:7-51``)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass
class LoraServingConfig:
    """The serving pipeline's shape: which encoder, which LoRA rank and targets,
    the batch geometry, device and dtype.  Every store, engine and task object is
    built from one instance of it.

    The encoder's dimensions (hidden size, layers, heads, FFN width, LayerNorm
    epsilon, activation) are read from the HuggingFace config of ``model_name``
    (``AutoConfig.from_pretrained``), or from ``hf_config`` when one is passed,
    so that a synthetic random-init encoder needs no checkpoint or network.
    """

    model_name: str
    lora_rank: int
    batch_size: int
    max_seq_len: int
    target_modules: list[str]
    device: torch.device
    dtype: torch.dtype
    hf_config: Any = None

    hidden_size: int = field(init=False)
    num_layers: int = field(init=False)
    num_heads: int = field(init=False)
    head_dim: int = field(init=False)
    intermediate_size: int = field(init=False)
    layer_norm_eps: float = field(init=False)
    hidden_act: str = field(init=False)

    def __post_init__(self):
        self.device = torch.device(self.device)
        hf = self.hf_config
        if hf is None:
            from transformers import AutoConfig

            hf = AutoConfig.from_pretrained(self.model_name)
            self.hf_config = hf
        self.hidden_size = hf.hidden_size
        self.num_layers = hf.num_hidden_layers
        self.num_heads = hf.num_attention_heads
        self.head_dim = hf.hidden_size // hf.num_attention_heads
        self.intermediate_size = hf.intermediate_size
        self.layer_norm_eps = hf.layer_norm_eps
        self.hidden_act = getattr(hf, "hidden_act", "gelu")
