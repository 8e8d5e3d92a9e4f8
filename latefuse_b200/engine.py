"""Encoders that apply per-row LoRA deltas with the native kernels.

Two engines, as in the reference:

* :class:`HFEncoderWithLora` (``engine="hf"``, the default) runs a stock
  HuggingFace ``AutoModel`` and adds each row's delta inside forward hooks on the
  targeted ``nn.Linear`` modules, in place on the projection output (the
  reference's hook does ``cat -> bmm -> bmm -> output + delta``,
  ``src/latefuse/model/hf_wrapper.py:169-219``).
* :class:`EncoderWithLora` (``engine="bert"``) is a BERT/RoBERTa/XLM-R encoder
  written for this path: one fused QKV GEMM per layer whose LoRA deltas for
  query/key/value come from one shrink pass over the shared input, then the
  expand adds into the fused output; the attention-output projection gets its
  own delta; attention runs through ``scaled_dot_product_attention``.  The
  reference's version (``src/latefuse/model/encoder.py``) skips ``dense``
  targets; this one applies them.

Both accept either a :class:`~latefuse_b200.batch.BatchLora` (slot ids; the
serving path) or the reference's ``list[LayerwiseBatchedWeights]``.
"""

from __future__ import annotations

import weakref

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.utils.hooks import RemovableHandle

from latefuse_b200.batch import BatchedLRWeights, BatchLora, LayerwiseBatchedWeights
from latefuse_b200.config import LoraServingConfig
from latefuse_b200.head import LRHeadOps, head_forward, head_forward_rows, pool_tokens, validate_pooling
from latefuse_b200.lora import (FactorCache, SegmentTable, blocked_u, fused_shrink_ok, linear_lora, lora_apply,
                                 lora_apply_into, lora_shrink_blocked, per_row_cache, workspace_bytes)
from latefuse_b200.encoder_ops import (ACT_GELU, add_layernorm, attention_varlen, embed_layernorm, gelu, linear,
                                       linear_accumulate)
from latefuse_b200.packing import PackedBatch, pack_rows

# Per-layer module paths (relative to "encoder.layer.{i}.") for each logical target.
# "dense" is the attention-output projection.
_TARGET_SUFFIXES: dict[str, dict[str, str]] = {
    "default": {
        "query": "attention.self.query",
        "key": "attention.self.key",
        "value": "attention.self.value",
        "dense": "attention.output.dense",
    },
    "deberta-v2": {
        "query": "attention.self.query_proj",
        "key": "attention.self.key_proj",
        "value": "attention.self.value_proj",
        "dense": "attention.output.dense",
    },
}


def _detach_hooks(handles: tuple[RemovableHandle, ...]) -> None:
    for handle in handles:
        handle.remove()


class _DeltaRunner:
    """Per-engine state for applying deltas: workspace, status word, and the
    conversion of the reference's layer-wise weight lists into factor caches."""

    def __init__(self, config: LoraServingConfig):
        self.config = config
        self._ws: Tensor | None = None
        self.status: Tensor | None = None

    def workspace(self, n_tokens: int, n_modules: int, device, dtype) -> Tensor:
        need = workspace_bytes(dtype, n_tokens, self.config.lora_rank, n_modules)
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        if self.status is None or self.status.device != device:
            self.status = torch.zeros(1, dtype=torch.int32, device=device)
        return self._ws

    @staticmethod
    def layerwise_cache(layer_w: LayerwiseBatchedWeights, module: str) -> FactorCache:
        a = torch.cat(layer_w.a[module], dim=0)
        b = torch.cat(layer_w.b[module], dim=0)
        return per_row_cache(a, b)


def _identity_segments(B: int, S: int, device) -> SegmentTable:
    return SegmentTable.for_padded(list(range(B)), S, device)


class HFEncoderWithLora(nn.Module):
    """Stock HF encoder with per-row LoRA deltas added in forward hooks (native kernels).

    Same constructor, ``encode_pooled`` / ``forward`` contract, hook guards and
    lifetime rules as the reference (``src/latefuse/model/hf_wrapper.py:56-370``).
    """

    def __init__(self, base: nn.Module, serving_config: LoraServingConfig):
        super().__init__()
        self.base = base
        self.config = serving_config
        self._runner = _DeltaRunner(serving_config)
        self._batch: BatchLora | list[LayerwiseBatchedWeights] | None = None
        self._segs: SegmentTable | None = None
        self._expected_shape: tuple[int, int, int] | None = None
        self._fired: set[tuple[int, str]] = set()
        self.shared_projection_skips = 0
        self._num_hooks = 0
        self._hook_handles: list[RemovableHandle] = []

        duplicates = sorted({t for t in serving_config.target_modules if serving_config.target_modules.count(t) > 1})
        if duplicates:
            raise ValueError(
                f"target_modules contains duplicate entries {duplicates}: {serving_config.target_modules}. "
                "Each projection may be hooked at most once."
            )
        suffixes = _TARGET_SUFFIXES.get(base.config.model_type, _TARGET_SUFFIXES["default"])
        modules = dict(base.named_modules())
        try:
            for logical in serving_config.target_modules:
                if logical not in suffixes:
                    raise ValueError(
                        f"target module '{logical}' has no mapping for model_type '{base.config.model_type}' "
                        f"(known: {sorted(suffixes)})"
                    )
                for layer_idx in range(serving_config.num_layers):
                    name = f"encoder.layer.{layer_idx}.{suffixes[logical]}"
                    if name not in modules:
                        raise ValueError(
                            f"module '{name}' not found in {base.config.model_type} model — cannot attach LoRA hook"
                        )
                    self._hook_handles.append(modules[name].register_forward_hook(self._make_hook(layer_idx, logical)))
                    self._num_hooks += 1
        except BaseException:
            _detach_hooks(tuple(self._hook_handles))
            self._hook_handles.clear()
            raise
        self._finalizer = weakref.finalize(self, _detach_hooks, tuple(self._hook_handles))
        self._finalizer.atexit = False

    def _make_hook(self, layer_idx: int, logical: str):
        key = (layer_idx, logical)
        wref = weakref.ref(self)  # no reference cycle through base's hook dicts

        def hook(module: nn.Module, inputs: tuple, output: Tensor):
            owner = wref()
            if owner is None or owner._batch is None:
                return None
            x = inputs[0]
            if key in owner._fired or x.shape != owner._expected_shape:
                owner.shared_projection_skips += 1
                return None
            owner._fired.add(key)
            owner._apply_delta(layer_idx, logical, x, output)
            return output

        return hook

    def _apply_delta(self, layer_idx: int, logical: str, x: Tensor, out: Tensor) -> None:
        batch = self._batch
        T = x.shape[0] * x.shape[1]
        ws = self._runner.workspace(T, 1, x.device, x.dtype)
        if isinstance(batch, BatchLora):
            store = batch.store
            cache = store.factor_cache(layer_idx)
            mod = store.module_index(logical)
            lora_apply(x, out, cache, batch.segments, [mod], [0], ws, self._runner.status)
        else:
            cache = _DeltaRunner.layerwise_cache(batch[layer_idx], logical)
            lora_apply(x, out, cache, self._segs, [0], [0], ws, self._runner.status)

    @classmethod
    def from_pretrained_serving(cls, serving_config: LoraServingConfig, attn_implementation: str | None = None):
        """Load the stock HF base model and attach LoRA hooks."""
        from transformers import AutoModel

        kwargs: dict = {"dtype": serving_config.dtype}
        if attn_implementation is not None:
            kwargs["attn_implementation"] = attn_implementation
        base = AutoModel.from_pretrained(serving_config.model_name, **kwargs)
        base.eval()
        return cls(base, serving_config).to(serving_config.device)

    def close(self) -> None:
        """Detach the LoRA hooks and drop the base model. Idempotent."""
        self._finalizer()
        self._hook_handles.clear()
        self.base = None

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        self.close()

    def encode_pooled(self, input_ids: Tensor, attention_mask: Tensor | None, lora_weights,
                      token_type_ids: Tensor | None = None, apply_lora: bool = True,
                      pooling: str = "auto") -> Tensor:
        """Base forward with LoRA deltas, up to the ``(B, H)`` pooled output.

        Raises ``RuntimeError`` if the adapter was not applied at every target
        projection, as the reference does.
        """
        validate_pooling(pooling)
        if self.base is None:
            raise RuntimeError(
                "this HFEncoderWithLora has been closed; its base model was released and it cannot run a "
                "forward pass. Build a new one with from_pretrained_serving()."
            )
        B, S = input_ids.shape
        cfg = self.config
        self._batch = lora_weights if apply_lora else None
        if apply_lora and not isinstance(lora_weights, BatchLora):
            self._segs = _identity_segments(B, S, input_ids.device)
        self._expected_shape = (B, S, cfg.hidden_size)
        self._fired = set()
        skips_before = self.shared_projection_skips
        try:
            kwargs = {}
            if token_type_ids is not None:
                kwargs["token_type_ids"] = token_type_ids
            out = self.base(input_ids=input_ids, attention_mask=attention_mask, **kwargs)
            fired = len(self._fired)
        finally:
            self._batch = None
            self._segs = None
            self._expected_shape = None
            self._fired = set()
        if apply_lora and fired != self._num_hooks:
            raise RuntimeError(
                f"LoRA hooks fired {fired}/{self._num_hooks} times on {self.base.config.model_type}: every target "
                f"projection was expected to be called on a tensor of shape {(B, S, cfg.hidden_size)}, and "
                f"{self.shared_projection_skips - skips_before} call(s) took the skip path instead. The base "
                "forward ran without the adapter delta, so anything measured from it would be wrong."
            )
        if pooling == "auto":
            pooled = getattr(out, "pooler_output", None)
            if pooled is None:
                pooled = out.last_hidden_state[:, 0]
            return pooled
        return pool_tokens(out.last_hidden_state, attention_mask, pooling)

    def forward(self, input_ids: Tensor, attention_mask: Tensor | None, lora_weights,
                lr_weights: BatchedLRWeights, output_lr: Tensor, token_type_ids: Tensor | None = None,
                apply_lora: bool = True, pooling: str = "auto") -> Tensor:
        """Encoder + batched per-tenant LR heads; fills ``output_lr (B, 1, max_labels)``."""
        pooled = self.encode_pooled(input_ids, attention_mask, lora_weights, token_type_ids, apply_lora, pooling)
        LRHeadOps.predict_proba(pooled.unsqueeze(1), lr_weights.coef, lr_weights.intercept, output_lr)
        return output_lr


# ---------------------------------------------------------------------------
# native encoder
# ---------------------------------------------------------------------------
_OFFSET_POSITION_TYPES = {"roberta", "xlm-roberta", "xlm-roberta-xl", "camembert", "mpnet"}
_QKV = ("query", "key", "value")


def varlen_attention(q: Tensor, k: Tensor, v: Tensor, cu_seqlens: Tensor, max_len: int) -> Tensor:
    """Non-causal attention of each packed sequence with itself, ``(T, heads, head_dim)``
    in and out, scale ``1/sqrt(head_dim)`` (FlashAttention's varlen forward)."""
    return torch.ops.aten._flash_attention_forward(q, k, v, cu_seqlens, cu_seqlens, max_len, max_len, 0.0,
                                                   False, False)[0]


def packed_mean(h: Tensor, pb: PackedBatch) -> Tensor:
    """Per-row mean of packed token states, with the reference's rounding points
    (``src/latefuse/ops/pooling.py:61-71``): the sum and the count are held in the
    model dtype, then divided."""
    acc = torch.zeros(pb.n_rows, h.shape[1], dtype=torch.float32, device=h.device)
    acc.index_add_(0, pb.row_of_token, h.float())
    counts = pb.row_lengths.to(h.dtype).clamp(min=1e-9)
    return acc.to(h.dtype) / counts.unsqueeze(1)


class _Layer(nn.Module):
    def __init__(self, H: int, I: int, eps: float):
        super().__init__()
        self.wqkv = nn.Parameter(torch.empty(3 * H, H))
        self.bqkv = nn.Parameter(torch.empty(3 * H))
        self.wo = nn.Parameter(torch.empty(H, H))
        self.bo = nn.Parameter(torch.empty(H))
        self.ln1 = nn.LayerNorm(H, eps=eps)
        self.wi = nn.Parameter(torch.empty(I, H))
        self.bi = nn.Parameter(torch.empty(I))
        self.wo2 = nn.Parameter(torch.empty(H, I))
        self.bo2 = nn.Parameter(torch.empty(H))
        self.ln2 = nn.LayerNorm(H, eps=eps)


class EncoderWithLora(nn.Module):
    """BERT-family encoder (BERT, RoBERTa, XLM-R, bge-m3 ...) with per-row LoRA deltas.

    Same ``encode_pooled`` / ``forward`` contract as the reference's
    ``EncoderWithLora`` (``src/latefuse/model/encoder.py:145-321``) and loads the
    same checkpoints (strictly: a checkpoint without a pooler is rejected, use the
    ``"hf"`` engine for those).
    """

    def __init__(self, hf_config, serving_config: LoraServingConfig):
        super().__init__()
        from transformers.activations import ACT2FN

        H, I = serving_config.hidden_size, serving_config.intermediate_size
        self.config = serving_config
        self.hf_config = hf_config
        self.num_heads = serving_config.num_heads
        self.head_dim = serving_config.head_dim
        self.eps = serving_config.layer_norm_eps
        self.pad_idx = hf_config.pad_token_id if hf_config.pad_token_id is not None else 0
        self.offset_positions = hf_config.model_type in _OFFSET_POSITION_TYPES
        self.word_embeddings = nn.Embedding(hf_config.vocab_size, H, padding_idx=hf_config.pad_token_id)
        self.position_embeddings = nn.Embedding(hf_config.max_position_embeddings, H)
        self.token_type_embeddings = nn.Embedding(max(1, hf_config.type_vocab_size), H)
        self.emb_ln = nn.LayerNorm(H, eps=self.eps)
        self.layers = nn.ModuleList([_Layer(H, I, self.eps) for _ in range(serving_config.num_layers)])
        self.pooler_w = nn.Parameter(torch.empty(H, H))
        self.pooler_b = nn.Parameter(torch.empty(H))
        self.act = ACT2FN[serving_config.hidden_act]
        #: the FFN activation is the exact (erf) GELU: run it on the native kernel
        self._native_gelu = serving_config.hidden_act == "gelu"
        self._runner = _DeltaRunner(serving_config)
        #: when a list, every LoRA delta op appends (start, end) CUDA events recorded
        #: around it on the current stream (used by the benchmark's roofline timing)
        self.lora_events: list | None = None
        #: compute the shrink inside the projection GEMM's launch where the kernel can
        #: (``lf_linear_lora_shrink``); False runs ``lf_lora_shrink_blocked`` first; or
        #: the set of projections to fuse (``{"qkv"}``, ``{"dense"}``)
        self.fuse_shrink: bool | set = True
        #: the LoRA'd projections read a (K, N) transposed copy of their weight (kept per
        #: weight, rebuilt when it changes), in the delta factors' operand form; off by
        #: default: it measured the same as the weight as given, at 8 MB more per layer
        self.kn_weights = False
        self._wt_cache: dict[int, tuple] = {}
        #: bf16/f16 FFN down projection on this library's GEMM accumulating onto its
        #: residual (``lf_linear_accumulate``) instead of torch's ``addmm_`` (cuBLAS,
        #: beta = 1).  Off by default: at the bge-m3 serving shape (17,410 tokens x 1,024
        #: x 4,096) cuBLAS's 240-token tiles fill the last wave that the 256-token CTA
        #: pair leaves 73% full (98 vs 103-109 us alone), and the serving step measured
        #: 0.45 ms faster with cuBLAS here.
        self.native_ffn_down = False
        targets = serving_config.target_modules
        self._qkv_targets = [(m, _QKV.index(m)) for m in targets if m in _QKV]
        self._dense_target = "dense" in targets
        unknown = sorted(set(targets) - set(_QKV) - {"dense"})
        if unknown:
            raise ValueError(f"target modules {unknown} have no mapping in the native encoder "
                             f"(known: {sorted(_QKV) + ['dense']})")

    # -- construction ----------------------------------------------------------
    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict[str, Tensor]) -> None:
        """Copy weights from a HuggingFace BERT-family state dict (strict)."""
        sd = {k.removeprefix("bert.").removeprefix("roberta."): v for k, v in sd.items()}
        used: set[str] = set()

        def take(key: str) -> Tensor:
            if key not in sd:
                hint = " — the checkpoint ships no pooler; use the HF hook engine ('hf')" if key.startswith("pooler.") else ""
                raise RuntimeError(f"{self.config.model_name} does not match the BERT-family layout: missing {key}{hint}")
            used.add(key)
            return sd[key]

        self.word_embeddings.weight.copy_(take("embeddings.word_embeddings.weight"))
        self.position_embeddings.weight.copy_(take("embeddings.position_embeddings.weight"))
        self.token_type_embeddings.weight.copy_(take("embeddings.token_type_embeddings.weight"))
        self.emb_ln.weight.copy_(take("embeddings.LayerNorm.weight"))
        self.emb_ln.bias.copy_(take("embeddings.LayerNorm.bias"))
        for i, layer in enumerate(self.layers):
            p = f"encoder.layer.{i}."
            layer.wqkv.copy_(torch.cat([take(p + f"attention.self.{m}.weight") for m in _QKV], 0))
            layer.bqkv.copy_(torch.cat([take(p + f"attention.self.{m}.bias") for m in _QKV], 0))
            layer.wo.copy_(take(p + "attention.output.dense.weight"))
            layer.bo.copy_(take(p + "attention.output.dense.bias"))
            layer.ln1.weight.copy_(take(p + "attention.output.LayerNorm.weight"))
            layer.ln1.bias.copy_(take(p + "attention.output.LayerNorm.bias"))
            layer.wi.copy_(take(p + "intermediate.dense.weight"))
            layer.bi.copy_(take(p + "intermediate.dense.bias"))
            layer.wo2.copy_(take(p + "output.dense.weight"))
            layer.bo2.copy_(take(p + "output.dense.bias"))
            layer.ln2.weight.copy_(take(p + "output.LayerNorm.weight"))
            layer.ln2.bias.copy_(take(p + "output.LayerNorm.bias"))
        self.pooler_w.copy_(take("pooler.dense.weight"))
        self.pooler_b.copy_(take("pooler.dense.bias"))
        ignorable = {"embeddings.position_ids", "embeddings.token_type_ids"}
        unexpected = sorted(k for k in sd if k not in used and k not in ignorable)
        if unexpected:
            raise RuntimeError(f"{self.config.model_name} does not match the BERT-family layout: unexpected={unexpected}")

    @classmethod
    def from_hf_model(cls, base: nn.Module, serving_config: LoraServingConfig) -> EncoderWithLora:
        model = cls(base.config, serving_config)
        model.load_hf_state_dict(base.state_dict())
        return model.to(device=serving_config.device, dtype=serving_config.dtype).eval()

    @classmethod
    def from_pretrained_serving(cls, serving_config: LoraServingConfig) -> EncoderWithLora:
        """Create the model and load base weights from HuggingFace."""
        from transformers import AutoModel

        base = AutoModel.from_pretrained(serving_config.model_name, dtype=serving_config.dtype)
        return cls.from_hf_model(base, serving_config)

    @classmethod
    @torch.no_grad()
    def random_init(cls, hf_config, serving_config: LoraServingConfig, seed: int = 0) -> EncoderWithLora:
        """A randomly initialised model (N(0, initializer_range) weights, zero biases, unit
        LayerNorms), drawn directly on the serving device: synthetic serving workloads."""
        model = cls(hf_config, serving_config).to(device=serving_config.device, dtype=serving_config.dtype)
        gen = torch.Generator(device=serving_config.device).manual_seed(seed)
        std = getattr(hf_config, "initializer_range", 0.02)
        ones = ("ln1.weight", "ln2.weight", "emb_ln.weight")
        zeros = ("ln1.bias", "ln2.bias", "emb_ln.bias", "bqkv", "bo", "bi", "bo2", "pooler_b")
        for name, p in model.named_parameters():
            if name.endswith(ones):
                p.fill_(1.0)
            elif name.split(".")[-1] in zeros or name.endswith(zeros[:3]):
                p.zero_()
            else:
                p.normal_(0.0, std, generator=gen)
        if hf_config.pad_token_id is not None:
            model.word_embeddings.weight[hf_config.pad_token_id].zero_()
        return model.eval()

    # -- forward -------------------------------------------------------------
    def position_ids(self, input_ids: Tensor) -> Tensor:
        """arange for BERT; mask-offset positions for the RoBERTa family (pad -> pad_idx)."""
        B, S = input_ids.shape
        if not self.offset_positions:
            return torch.arange(S, device=input_ids.device).unsqueeze(0).expand(B, -1)
        mask = input_ids.ne(self.pad_idx).int()
        return (torch.cumsum(mask, dim=1) * mask).long() + self.pad_idx

    def _resolve(self, lora_weights, B: int, S: int, device):
        """(per-layer cache getter, segment table) for this batch."""
        if isinstance(lora_weights, BatchLora):
            store = lora_weights.store
            qkv_idx = [store.module_index(m) for m, _ in self._qkv_targets]
            dense_idx = [store.module_index("dense")] if self._dense_target else []
            return (lambda l, _m=None: store.factor_cache(l)), lora_weights.segments, qkv_idx, dense_idx, True
        segs = _identity_segments(B, S, device)
        return None, segs, None, None, False

    def _event_pair(self, kind: str):
        if self.lora_events is None:
            return None
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        self.lora_events.append((kind, start, end))
        return start, end

    def encode_pooled(self, input_ids: Tensor, attention_mask: Tensor | None, lora_weights,
                      token_type_ids: Tensor | None = None, apply_lora: bool = True,
                      pooling: str = "auto") -> Tensor:
        """Base forward with LoRA deltas, up to the ``(B, H)`` pooled output."""
        validate_pooling(pooling)
        hidden = self.encode(input_ids, attention_mask, lora_weights, token_type_ids, apply_lora)
        if pooling == "auto":
            return torch.tanh(F.linear(hidden[:, 0], self.pooler_w, self.pooler_b))
        return pool_tokens(hidden, attention_mask, pooling)

    def encode(self, input_ids: Tensor, attention_mask: Tensor | None, lora_weights,
               token_type_ids: Tensor | None = None, apply_lora: bool = True) -> Tensor:
        """Final hidden states ``(B, S, H)``."""
        B, S = input_ids.shape
        H, nh, hd = self.config.hidden_size, self.num_heads, self.head_dim
        dev = input_ids.device
        T = B * S
        if token_type_ids is None:
            token_type_ids = torch.zeros(B, S, dtype=torch.long, device=dev)
        x = self.word_embeddings(input_ids) + self.token_type_embeddings(token_type_ids)
        h = add_layernorm(x, self.position_embeddings(self.position_ids(input_ids)), self.emb_ln.weight,
                          self.emb_ln.bias, self.eps).view(T, H)

        attn_mask = None
        if attention_mask is not None:
            attn_mask = attention_mask.to(torch.bool).view(B, 1, 1, S)

        do_lora = apply_lora and (self._qkv_targets or self._dense_target)
        if do_lora:
            getter, segs, qkv_idx, dense_idx, sloted = self._resolve(lora_weights, B, S, dev)
            n_mod = max(1, len(self._qkv_targets))
            ws = self._runner.workspace(T, n_mod, dev, h.dtype)
            status = self._runner.status
            qkv_offs = [j * H for _, j in self._qkv_targets]

        for l, layer in enumerate(self.layers):
            qkv = F.linear(h, layer.wqkv, layer.bqkv)  # (T, 3H)
            if do_lora and self._qkv_targets:
                if sloted:
                    ev = self._event_pair("qkv")
                    lora_apply(h, qkv, getter(l), segs, qkv_idx, qkv_offs, ws, status)
                    if ev is not None:
                        ev[1].record()
                else:
                    for (m, j) in self._qkv_targets:
                        cache = _DeltaRunner.layerwise_cache(lora_weights[l], m)
                        lora_apply(h, qkv, cache, segs, [0], [j * H], ws, status)
            q, k, v = qkv.view(B, S, 3, nh, hd).permute(2, 0, 3, 1, 4).unbind(0)
            ctx = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)
            ctx = ctx.transpose(1, 2).reshape(T, H)
            ao = F.linear(ctx, layer.wo, layer.bo)
            if do_lora and self._dense_target:
                if sloted:
                    ev = self._event_pair("dense")
                    lora_apply(ctx, ao, getter(l), segs, dense_idx, [0], ws, status)
                    if ev is not None:
                        ev[1].record()
                else:
                    cache = _DeltaRunner.layerwise_cache(lora_weights[l], "dense")
                    lora_apply(ctx, ao, cache, segs, [0], [0], ws, status)
            h = self._ffn(layer, ao, h)
        return h.view(B, S, H)

    def _ffn(self, layer: _Layer, ao: Tensor, h: Tensor | None) -> Tensor:
        """``h1 = LN1(ao + h)`` (``LN1(ao)`` when ``h`` is None: the residual is already
        in ``ao``), then ``LN2(W2 act(W1 h1) + b2 + h1)``, on the native add+LayerNorm and
        GELU kernels.  For bf16/f16 the up projection and its exact GELU run as one launch
        of this library's tcgen05 GEMM (the GELU in its epilogue), the down projection
        accumulates onto ``h1`` in place (beta = 1: cuBLAS, or this library's GEMM when
        ``native_ffn_down``; ``h1`` is not read again) and LayerNorm adds ``b2``, so the
        residual is not read a second time."""
        h1 = add_layernorm(ao, h, layer.ln1.weight, layer.ln1.bias, self.eps)
        if self._native_gelu and self._gemm_ok(h1.dtype, layer.wi.shape):
            mid = linear(h1, layer.wi, layer.bi, act=ACT_GELU)
        else:
            mid = F.linear(h1, layer.wi, layer.bi)
            mid = gelu(mid, out=mid) if self._native_gelu else self.act(mid)
        if h1.dtype in (torch.bfloat16, torch.float16):
            if self.native_ffn_down and self._gemm_ok(h1.dtype, layer.wo2.shape):
                linear_accumulate(mid, layer.wo2, h1)
            else:
                h1.view(-1, h1.shape[-1]).addmm_(mid.view(-1, mid.shape[-1]), layer.wo2.t())
            return add_layernorm(h1, None, layer.ln2.weight, layer.ln2.bias, self.eps, out=h1, vec=layer.bo2)
        o = F.linear(mid, layer.wo2, layer.bo2)
        return add_layernorm(o, h1, layer.ln2.weight, layer.ln2.bias, self.eps, out=o)

    def _transposed(self, w: Tensor) -> Tensor | None:
        """``w``'s ``(K, N)`` transpose for :func:`linear_lora` (None when ``kn_weights`` is
        off), cached per weight and rebuilt when the weight is replaced or changed in place."""
        if not self.kn_weights:
            return None
        hit = self._wt_cache.get(id(w))
        if hit is not None and hit[1] == w._version and hit[2] == w.data_ptr():
            return hit[0]
        t = w.detach().t().contiguous()
        self._wt_cache[id(w)] = (t, w._version, w.data_ptr())
        return t

    @staticmethod
    def _gemm_ok(dtype: torch.dtype, weight_shape) -> bool:
        """Whether this library's GEMM (``lf_linear``) takes a projection of this weight:
        bf16/f16, output width a multiple of 256, input width a multiple of 64."""
        n, k = weight_shape
        return dtype in (torch.bfloat16, torch.float16) and n % 256 == 0 and k % 64 == 0

    def _lora_gemm_ok(self, dtype: torch.dtype, rank: int) -> bool:
        """Whether the packed forward runs the LoRA'd projections on this library's
        GEMM with the delta in its accumulator (``linear_lora``)."""
        return dtype in (torch.bfloat16, torch.float16) and self.config.hidden_size % 256 == 0 and \
            rank in (16, 32, 64)

    def _fused_dense_ok(self, dtype: torch.dtype, rank: int) -> bool:
        """Whether the packed forward writes the attention-output delta (with bias and
        residual) first and lets the projection GEMM accumulate onto it
        (``lora_apply_into``).  Not done for q/k/v: there the in-place delta right
        after the GEMM re-reads an output the L2 still holds, which measured faster
        than writing the delta to a fresh buffer for the GEMM to read."""
        return bool(self._dense_target) and dtype in (torch.bfloat16, torch.float16) and \
            self.config.hidden_size % 128 == 0 and rank in (8, 16, 32, 64)

    # -- padding-free forward ------------------------------------------------
    @property
    def supports_packing(self) -> bool:
        """Whether :meth:`encode_pooled_packed` can run: FlashAttention's varlen
        kernel takes f16/bf16 with head_dim a multiple of 8 up to 256."""
        return (self.config.dtype in (torch.float16, torch.bfloat16) and self.head_dim % 8 == 0
                and self.head_dim <= 256)

    def pack(self, input_ids: Tensor, lengths: list[int], slots: list[int],
             token_type_ids: Tensor | None = None) -> PackedBatch:
        """Pack right-padded host rows (``lengths[b]`` real tokens first) for
        :meth:`encode_pooled_packed`; position ids follow the padded rows."""
        return pack_rows(input_ids, lengths, slots, self.pad_idx if self.offset_positions else None,
                         token_type_ids, self.config.device)

    def encode_packed(self, pb: PackedBatch, store, apply_lora: bool = True) -> Tensor:
        """Final hidden states of the real tokens, ``(n_tokens, H)`` in packed order.

        Same per-token arithmetic as :meth:`encode`; attention runs per sequence
        (the tcgen05 kernel ``lf_attention_varlen`` for head_dim 64, FlashAttention
        varlen otherwise), so no padded key exists.
        ``store`` is the :class:`~latefuse_b200.store.AdapterStore` whose slots
        ``pb.segments`` names.
        """
        T = pb.n_tokens
        H, nh, hd = self.config.hidden_size, self.num_heads, self.head_dim
        if self._runner.status is None or self._runner.status.device != pb.ids.device:
            self._runner.status = torch.zeros(1, dtype=torch.int32, device=pb.ids.device)
        if H % 8 == 0 and H <= 4096:  # gathers, both adds and the LayerNorm in one launch
            h = embed_layernorm(pb.ids, pb.positions, pb.token_types, self.word_embeddings.weight,
                                self.position_embeddings.weight, self.token_type_embeddings.weight,
                                self.emb_ln.weight, self.emb_ln.bias, self.eps, status=self._runner.status)
        else:
            x = self.word_embeddings(pb.ids) + self.token_type_embeddings(pb.token_types)
            h = add_layernorm(x, self.position_embeddings(pb.positions), self.emb_ln.weight, self.emb_ln.bias,
                              self.eps)

        do_lora = apply_lora and store is not None and (self._qkv_targets or self._dense_target)
        if do_lora:
            qkv_idx = [store.module_index(m) for m, _ in self._qkv_targets]
            dense_idx = [store.module_index("dense")] if self._dense_target else []
            ws = self._runner.workspace(T, max(1, len(self._qkv_targets)), h.device, h.dtype)
            status = self._runner.status
            qkv_offs = [j * H for _, j in self._qkv_targets]
            segs = pb.segments
            rank = store.factor_cache(0).rank
            # q/k/v and the attention output on the tcgen05 GEMM with the delta in
            # its accumulator (shrink first, into (tile, segment) blocks of u)
            gemm_ok = self._lora_gemm_ok(h.dtype, rank) and segs.use_records
            gemm_qkv = gemm_ok and sorted(j for _, j in self._qkv_targets) == [0, 1, 2]
            qkv_by_col = [store.module_index(m) for m, _ in sorted(self._qkv_targets, key=lambda t: t[1])]
            gemm_dense = gemm_ok and bool(self._dense_target)
            fuse_dense = not gemm_dense and self._fused_dense_ok(h.dtype, rank)
            if gemm_qkv:
                u_qkv = blocked_u(3, T, segs.n_segs, rank, h.dtype, h.device)
            if gemm_dense:
                u_dense = blocked_u(1, T, segs.n_segs, rank, h.dtype, h.device)
            fuse = self.fuse_shrink if isinstance(self.fuse_shrink, (set, frozenset)) else \
                ({"qkv", "dense"} if self.fuse_shrink else set())
            fuse_qkv = gemm_qkv and "qkv" in fuse and fused_shrink_ok(qkv_by_col, rank)
            fuse_dense_shrink = gemm_dense and "dense" in fuse and fused_shrink_ok(dense_idx, rank)
        else:
            fuse_dense = gemm_qkv = gemm_dense = fuse_qkv = fuse_dense_shrink = False

        for l, layer in enumerate(self.layers):
            if gemm_qkv:
                cache = store.factor_cache(l)
                if not fuse_qkv:
                    ev = self._event_pair("qkv_shrink")
                    lora_shrink_blocked(h, u_qkv, cache, segs, qkv_by_col, status)
                    if ev is not None:
                        ev[1].record()
                ev = self._event_pair("qkv_gemm")
                qkv = linear_lora(h, layer.wqkv, layer.bqkv, u_qkv, cache, segs, qkv_by_col, H, status=status,
                                  shrink=fuse_qkv, weight_t=self._transposed(layer.wqkv))
                if ev is not None:
                    ev[1].record()
            else:
                qkv = F.linear(h, layer.wqkv, layer.bqkv)  # (T, 3H)
                if do_lora and self._qkv_targets:
                    ev = self._event_pair("qkv")
                    lora_apply(h, qkv, store.factor_cache(l), segs, qkv_idx, qkv_offs, ws, status)
                    if ev is not None:
                        ev[1].record()
            if hd == 64:
                ctx = attention_varlen(qkv, nh, pb.attn_items, hd ** -0.5, status=self._runner.status)
            else:  # head sizes the tcgen05 kernel does not tile
                q, k, v = qkv.view(T, 3, nh, hd).unbind(1)
                ctx = varlen_attention(q, k, v, pb.cu_seqlens, pb.max_len).view(T, H)
            if gemm_dense:
                cache = store.factor_cache(l)
                if not fuse_dense_shrink:
                    ev = self._event_pair("dense_shrink")
                    lora_shrink_blocked(ctx, u_dense, cache, segs, dense_idx, status)
                    if ev is not None:
                        ev[1].record()
                ev = self._event_pair("dense_gemm")
                ao = linear_lora(ctx, layer.wo, layer.bo, u_dense, cache, segs, dense_idx, H, status=status,
                                 shrink=fuse_dense_shrink, weight_t=self._transposed(layer.wo))
                if ev is not None:
                    ev[1].record()
                h = self._ffn(layer, ao, h)
            elif fuse_dense:
                # The delta, bias and residual go first, into a fresh output that
                # the projection GEMM accumulates onto (beta = 1); the LayerNorm
                # then reads one tensor instead of two.
                ev = self._event_pair("dense")
                ao = torch.empty(T, H, dtype=h.dtype, device=h.device)
                lora_apply_into(ctx, ao, store.factor_cache(l), segs, dense_idx, [0], ws, status,
                                residual=h, bias=layer.bo)
                if ev is not None:
                    ev[1].record()
                ao.addmm_(ctx, layer.wo.t())
                h = self._ffn(layer, ao, None)
            else:
                ao = F.linear(ctx, layer.wo, layer.bo)
                if do_lora and self._dense_target:
                    ev = self._event_pair("dense")
                    lora_apply(ctx, ao, store.factor_cache(l), segs, dense_idx, [0], ws, status)
                    if ev is not None:
                        ev[1].record()
                h = self._ffn(layer, ao, h)
        return h

    def encode_pooled_packed(self, pb: PackedBatch, store, pooling: str = "auto",
                             apply_lora: bool = True) -> Tensor:
        """Pooled ``(B, H)`` rows in input order from a packed batch."""
        validate_pooling(pooling)
        h = self.encode_packed(pb, store, apply_lora)
        return self.heads_packed(h, pb, pooling)

    def heads_packed(self, h: Tensor, pb: PackedBatch, pooling: str, *, coef: Tensor | None = None,
                     bias: Tensor | None = None, head_table: Tensor | None = None, n_max: int = 0,
                     logits_out: Tensor | None = None, probs_out: Tensor | None = None) -> Tensor:
        """The pooled ``(B, H)`` rows of packed hidden states ``h`` and, given a head
        table, the per-tenant logits and probabilities, in one native call for CLS
        and ``"auto"`` pooling (row gather -> pooler -> head -> softmax,
        ``lf_head_forward_rows``)."""
        B, H = pb.n_rows, h.shape[1]
        pooled = torch.empty(B, H, dtype=h.dtype, device=h.device)
        head = dict(coef=coef, bias=bias, head_table=head_table, n_max=n_max, logits_out=logits_out,
                    probs_out=probs_out, status=self._runner.status)
        if pooling == "mean":
            pooled = packed_mean(h, pb)
            if coef is not None:
                head_forward(pooled, pooling="none", **head)
            return pooled
        pooler = dict(pooler_w=self.pooler_w, pooler_b=self.pooler_b) if pooling == "auto" else {}
        head_forward_rows(h, pb.first_token, pooled_out=pooled, **pooler, **head)
        return pooled

    def forward(self, input_ids: Tensor, attention_mask: Tensor | None, lora_weights,
                lr_weights: BatchedLRWeights, output_lr: Tensor, token_type_ids: Tensor | None = None,
                apply_lora: bool = True, pooling: str = "auto") -> Tensor:
        """Full mixed-tenant forward: encoder + batched per-tenant LR heads."""
        pooled = self.encode_pooled(input_ids, attention_mask, lora_weights, token_type_ids, apply_lora, pooling)
        LRHeadOps.predict_proba(pooled.unsqueeze(1), lr_weights.coef, lr_weights.intercept, output_lr)
        return output_lr
