"""Oracle for the encoder forward with per-row LoRA deltas (the reference's "hf" engine).

Restates ``HFEncoderWithLora`` (``src/latefuse/model/hf_wrapper.py:81-342``): a
stock HuggingFace model whose targeted projections get, in a forward hook,

    a = cat(per-row A[layer]);  b = cat(per-row B[layer])           (:212-214)
    return output + bmm(bmm(x, a), b)   (shrink/expand in the dtype) (:215-217)

and the pooling of ``encode_pooled`` (``:337-342``).  ``dense`` maps to the
attention-output projection ``attention.output.dense`` (the reference maps only
query/key/value; adding the entry is how its own hooks are pointed at it).
"""

from __future__ import annotations

import torch
from torch import Tensor

from oracle.head import pool_tokens
from oracle.lora import lora_delta

SUFFIXES = {
    "query": "attention.self.query",
    "key": "attention.self.key",
    "value": "attention.self.value",
    "dense": "attention.output.dense",
}


class HookedEncoder:
    """A HuggingFace encoder with the reference's per-row LoRA hooks attached.

    ``adapters[tenant] = {"wa": {m: (L,H,R)}, "wb": {m: (L,R,H)}}``.
    """

    def __init__(self, base, adapters: dict, targets: list[str]):
        self.base = base
        self.adapters = adapters
        self.targets = list(targets)
        self._rows: list[str] | None = None
        self._handles = []
        modules = dict(base.named_modules())
        for m in self.targets:
            for layer in range(base.config.num_hidden_layers):
                mod = modules[f"encoder.layer.{layer}.{SUFFIXES[m]}"]
                self._handles.append(mod.register_forward_hook(self._hook(layer, m)))

    def _hook(self, layer: int, module: str):
        def hook(_mod, inputs, output):
            if self._rows is None:
                return None
            x = inputs[0]
            dt = output.dtype
            a = torch.stack([self.adapters[t]["wa"][module][layer] for t in self._rows]).to(x.device, dt)
            b = torch.stack([self.adapters[t]["wb"][module][layer] for t in self._rows]).to(x.device, dt)
            d = lora_delta(x.to(dt), a, b)
            return (output.float() + d.float()).to(dt)

        return hook

    @torch.no_grad()
    def encode_pooled(self, input_ids: Tensor, attention_mask: Tensor | None, tenants: list[str],
                      pooling: str = "cls", apply_lora: bool = True, token_type_ids: Tensor | None = None) -> Tensor:
        self._rows = list(tenants) if apply_lora else None
        try:
            kw = {} if token_type_ids is None else {"token_type_ids": token_type_ids}
            out = self.base(input_ids=input_ids, attention_mask=attention_mask, **kw)
        finally:
            self._rows = None
        if pooling == "auto":
            pooled = getattr(out, "pooler_output", None)
            return out.last_hidden_state[:, 0] if pooled is None else pooled
        return pool_tokens(out.last_hidden_state, attention_mask, pooling)

    def close(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()


def build_model(config_cls, model_cls, conf: dict, state: dict | None = None, dtype=torch.float32, seed: int = 0):
    """A seeded (or state-dict-loaded) HuggingFace model on the CPU, in eval mode."""
    torch.manual_seed(seed)
    model = model_cls(config_cls(**conf)).eval()
    if state is not None:
        model.load_state_dict(state)
    return model.to(dtype)
