"""Load adapters trained with HuggingFace PEFT (mirror of ``src/latefuse/loaders.py``)."""

from __future__ import annotations

import json
import os

import torch

from latefuse_b200.engine import _TARGET_SUFFIXES
from latefuse_b200.store import AdapterStore

_WEIGHT_FILES = ("adapter_model.safetensors", "adapter_model.bin")


def peft_key_fn(model_type: str, adapter_name: str = "default"):
    """``(layer_idx, module) -> (key_A, key_B)`` for PEFT's state-dict naming on ``model_type``."""
    suffixes = _TARGET_SUFFIXES.get(model_type, _TARGET_SUFFIXES["default"])
    infix = "" if adapter_name in (None, "", "default") else f".{adapter_name}"

    def key_fn(layer_idx: int, module: str) -> tuple[str, str]:
        if module not in suffixes:
            raise ValueError(f"target module '{module}' has no mapping for model_type '{model_type}' "
                             f"(known: {sorted(suffixes)})")
        stem = f"base_model.model.encoder.layer.{layer_idx}.{suffixes[module]}.lora_"
        return f"{stem}A{infix}.weight", f"{stem}B{infix}.weight"

    return key_fn


def _read_state_dict(path: str, device) -> dict:
    if os.path.isdir(path):
        for name in _WEIGHT_FILES:
            candidate = os.path.join(path, name)
            if os.path.exists(candidate):
                return _read_state_dict(candidate, device)
        raise FileNotFoundError(f"{path} holds none of {list(_WEIGHT_FILES)}; expected a PEFT adapter directory")
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file

        return load_file(path, device=str(device))
    return torch.load(path, map_location=device, weights_only=True)


def load_peft_adapter(store: AdapterStore, adapter_id: str, path: str, *, adapter_name: str = "default",
                      lora_alpha: float | None = None, strict: bool = True, pad_rank: bool = False) -> None:
    """Load a PEFT adapter directory into ``store`` under ``adapter_id``.

    Checks ``adapter_config.json`` against the serving config (rank, target
    modules) and folds ``lora_alpha / r`` into B, as the reference does.  With
    ``pad_rank`` an adapter trained at a lower rank than the store's is accepted
    and zero-padded into its slot (mixed-rank serving; same delta).

    Raises:
        ValueError:        on a config mismatch under ``strict``.
        FileNotFoundError: if no weights file is found.
        KeyError:          if the state dict lacks an expected layer key.
    """
    cfg = store.config
    directory = path if os.path.isdir(path) else os.path.dirname(path) or "."
    peft_config_path = os.path.join(directory, "adapter_config.json")
    peft_config: dict = {}
    if os.path.exists(peft_config_path):
        with open(peft_config_path) as fh:
            peft_config = json.load(fh)
    if peft_config:
        _check_compatible(peft_config, cfg, adapter_id, strict, pad_rank)
    if lora_alpha is None:
        lora_alpha = peft_config.get("lora_alpha")
    model_type = cfg.hf_config.model_type
    state_dict = _read_state_dict(path, "cpu" if cfg.device.type != "cuda" else cfg.device)
    store.load_from_state_dict(adapter_id, state_dict, peft_key_fn(model_type, adapter_name), lora_alpha=lora_alpha,
                               pad_rank=pad_rank or not strict)


def _check_compatible(peft_config: dict, cfg, adapter_id: str, strict: bool, pad_rank: bool = False) -> None:
    import warnings

    problems = []
    rank = peft_config.get("r")
    if rank is not None and rank != cfg.lora_rank and not (pad_rank and rank < cfg.lora_rank):
        problems.append(
            f"adapter was trained at rank {rank} but this pipeline serves rank {cfg.lora_rank}. One pipeline "
            "serves one rank; build a second pipeline for the other."
        )
    targets = peft_config.get("target_modules")
    if targets is not None:
        trained = {str(t).removesuffix("_proj") for t in targets}
        served = {str(t).removesuffix("_proj") for t in cfg.target_modules}
        if trained != served:
            problems.append(
                f"adapter targets {sorted(trained)} but this pipeline adapts {sorted(served)}. Serving it would "
                "apply the deltas to the wrong projections."
            )
    if not problems:
        return
    message = f"adapter '{adapter_id}' does not match the serving config: " + " ".join(problems)
    if strict:
        raise ValueError(message + " Pass strict=False to load anyway.")
    warnings.warn(message, stacklevel=3)
