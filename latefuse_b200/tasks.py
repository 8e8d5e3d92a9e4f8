"""Task-level API (mirror of ``src/latefuse/tasks/*``): what a user calls.

``TaskPipeline`` owns tokenizer, engine, adapter store and assembler and turns
request lists of any length into fixed ``batch_size`` x ``max_seq_len``
forward passes (``src/latefuse/tasks/base.py``).  The wrappers add embeddings
(L2-normalised), classification with per-tenant heads, and cross-encoder
reranking on top.  Differences from the reference, all invisible in results:
tenant ids map to cache slots instead of gathered weights; padded positions of
right-padded rows get no LoRA delta (``skip_padding``), and with the native
encoder they are not computed at all (``pack_tokens``: real tokens only, rows
grouped by tenant, attention per sequence); softmax/sigmoid of the heads run on
the GPU next to the head GEMV.
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from dataclasses import dataclass
from typing import TypeVar

import numpy as np
import torch
from torch import Tensor

from latefuse_b200.batch import BatchAssembler, IndexSelectBatchAssembler
from latefuse_b200.config import LoraServingConfig
from latefuse_b200.engine import EncoderWithLora, HFEncoderWithLora
from latefuse_b200.head import head_forward, l2_normalize, validate_pooling
from latefuse_b200.heads import HeadStore
from latefuse_b200.rank_buckets import store_for_batch
from latefuse_b200.store import AdapterStore

T = TypeVar("T")

#: ``"hf"`` hooks a stock HuggingFace ``AutoModel``; ``"bert"`` is the native BERT-family encoder.
ENGINES = ("hf", "bert")

#: Accepted assembler names; both serve from the slot cache.
ASSEMBLERS = ("cpu", "index_select")


def chunk_and_pad(items: Sequence[T], batch_size: int) -> Iterator[tuple[list[T], int]]:
    """Yield ``(chunk, n_valid)`` where every chunk has exactly ``batch_size`` entries.

    The last chunk is padded by repeating its last real item
    (``src/latefuse/tasks/batching.py:23-52``); callers slice results to ``n_valid``.
    """
    if batch_size <= 0:
        raise ValueError(f"batch_size must be positive, got {batch_size}")
    for start in range(0, len(items), batch_size):
        chunk = list(items[start : start + batch_size])
        n_valid = len(chunk)
        if n_valid < batch_size:
            chunk.extend([chunk[-1]] * (batch_size - n_valid))
        yield chunk, n_valid


def stream_to_host(step, batches, depth: int = 2) -> Iterator[Tensor]:
    """Run ``step(*batch)`` (queues device work, returns a device tensor) over
    ``batches`` with up to ``depth`` batches in flight, yielding each result as a pinned
    host tensor in batch order.  With ``depth`` 2 the host packs, copies and launches
    batch i + 1 while the device computes batch i, so host preparation stops adding to
    the step time; ``depth`` 1 waits for every batch before starting the next."""
    from collections import deque

    if depth < 1:
        raise ValueError(f"depth must be at least 1, got {depth}")
    pending: deque = deque()
    for batch in batches:
        out = step(*batch)
        host = torch.empty(out.shape, dtype=out.dtype, pin_memory=out.is_cuda)
        host.copy_(out, non_blocking=out.is_cuda)
        done = None
        if out.is_cuda:
            done = torch.cuda.Event()
            done.record()
        pending.append((host, done))
        if len(pending) >= depth:
            host, done = pending.popleft()
            if done is not None:
                done.synchronize()
            yield host
    while pending:
        host, done = pending.popleft()
        if done is not None:
            done.synchronize()
        yield host


def _default_device() -> torch.device:
    return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")


def _default_dtype(device: torch.device) -> torch.dtype:
    return torch.float16 if device.type == "cuda" else torch.float32


def right_padded_lengths(mask: Tensor) -> list[int] | None:
    """Per-row real lengths of a host ``(B, S)`` 0/1 mask, or None unless every row is
    ones followed by zeros (only then can padding be skipped as a suffix)."""
    m = mask.numpy() if mask.dtype != torch.bool else mask.numpy().astype(np.int8)
    if m.ndim != 2 or m.size == 0:
        return None if m.ndim != 2 else [0] * m.shape[0]
    # ones followed by zeros: 0/1 values, never increasing along a row
    if ((m != 0) & (m != 1)).any() or (m[:, 1:] > m[:, :-1]).any():
        return None
    return m.sum(axis=1).astype(np.int64).tolist()


class TaskPipeline:
    """Base class: tokenize, assemble, encode, drop padding."""

    def __init__(self, config: LoraServingConfig, *, engine: str = "hf", assembler: str = "cpu",
                 pooling: str = "auto", tokenizer=None, model=None, store: AdapterStore | None = None,
                 skip_padding: bool = True, pack_tokens: bool = True):
        if engine not in ENGINES:
            raise ValueError(f"unknown engine {engine!r}; expected one of {', '.join(map(repr, ENGINES))}")
        if assembler not in ASSEMBLERS:
            raise ValueError(f"unknown assembler {assembler!r}; expected one of {', '.join(map(repr, ASSEMBLERS))}")
        validate_pooling(pooling)
        self.config = config
        self.pooling = pooling
        self.skip_padding = skip_padding
        self.pack_tokens = pack_tokens
        self._tokenizer = tokenizer
        if model is None:
            cls = HFEncoderWithLora if engine == "hf" else EncoderWithLora
            model = cls.from_pretrained_serving(config)
        self.model = model.eval()
        self.store = store if store is not None else AdapterStore(config)
        self._assembler_kind = assembler
        self._assembler = None

    @property
    def tokenizer(self):
        """The HF tokenizer of ``model_name`` (loaded on first use; pre-tokenized calls never need it)."""
        if self._tokenizer is None:
            from transformers import AutoTokenizer

            self._tokenizer = AutoTokenizer.from_pretrained(self.config.model_name)
        return self._tokenizer

    @tokenizer.setter
    def tokenizer(self, value) -> None:
        self._tokenizer = value

    @classmethod
    def from_pretrained(cls, model_name: str, *, lora_rank: int = 8, batch_size: int = 32,
                        max_seq_len: int = 128, target_modules: Sequence[str] = ("query", "value"),
                        device: torch.device | str | None = None, dtype: torch.dtype | None = None,
                        engine: str = "hf", assembler: str = "cpu", pooling: str = "auto", **kwargs):
        """Build a pipeline from a HuggingFace model id or local directory."""
        device = torch.device(device) if device is not None else _default_device()
        dtype = dtype if dtype is not None else _default_dtype(device)
        config = LoraServingConfig(model_name=model_name, lora_rank=lora_rank, batch_size=batch_size,
                                   max_seq_len=max_seq_len, target_modules=list(target_modules), device=device,
                                   dtype=dtype)
        return cls(config, engine=engine, assembler=assembler, pooling=pooling, **kwargs)

    # -- adapters ------------------------------------------------------------
    def register_adapter(self, tenant_id: str, path: str, **kwargs) -> None:
        """Make a trained PEFT adapter resident under ``tenant_id``."""
        from latefuse_b200.loaders import load_peft_adapter

        load_peft_adapter(self.store, tenant_id, path, **kwargs)
        self._invalidate_assembler()

    def register_synthetic(self, tenant_id: str, seed: int | None = None) -> None:
        """Make a randomly-initialised adapter resident. For benchmarking and tests."""
        self.store.load_synthetic(tenant_id, seed=seed)
        self._invalidate_assembler()

    def evict_adapter(self, tenant_id: str) -> None:
        self.store.evict(tenant_id)
        self._invalidate_assembler()

    @property
    def tenant_ids(self) -> list[str]:
        return self.store.adapter_ids()

    # -- internals -------------------------------------------------------------
    def _invalidate_assembler(self) -> None:
        """Drop the assembler after the store changes (cheap: it holds only views)."""
        self._assembler = None

    def _get_assembler(self):
        if self._assembler is None:
            kind = IndexSelectBatchAssembler if self._assembler_kind == "index_select" else BatchAssembler
            self._assembler = kind(self.store, self.config)
        return self._assembler

    def _tokenize(self, texts: list[str], text_pairs: list[str] | None):
        cfg = self.config
        args = (texts,) if text_pairs is None else (texts, text_pairs)
        return self.tokenizer(*args, padding="max_length", truncation=True, max_length=cfg.max_seq_len,
                              return_tensors="pt")

    def encode_tokens(self, input_ids: Tensor, attention_mask: Tensor | None, tenants: Sequence[str],
                      token_type_ids: Tensor | None = None, pooling: str | None = None,
                      head: dict | None = None) -> Tensor:
        """Pooled ``(B, H)`` rows for one pre-tokenized batch (host or device tensors).

        Host tensors are copied to the device here (pinned, asynchronous).  With
        ``head`` (the keyword arguments of :func:`~latefuse_b200.head.head_forward`'s
        head: coef, bias, head_table, n_max, logits_out, probs_out) the per-tenant
        heads run too; on the padding-free path the row gather, pooler, head and
        softmax are then one native call.
        """
        pooling = validate_pooling(pooling or self.pooling)
        cfg = self.config
        if len(tenants) != input_ids.shape[0]:
            raise ValueError(f"got {input_ids.shape[0]} rows but {len(tenants)} tenant ids")
        lengths = None
        if self.skip_padding and attention_mask is not None and attention_mask.device.type == "cpu":
            lengths = right_padded_lengths(attention_mask)
        packable = (self.pack_tokens and lengths is not None and min(lengths, default=0) >= 1
                    and input_ids.device.type == "cpu"
                    and (token_type_ids is None or token_type_ids.device.type == "cpu")
                    and getattr(self.model, "supports_packing", False))
        # a store of native-rank buckets serves each batch from its r_max staging cache
        store = store_for_batch(self.store, list(tenants))
        if packable:
            # padding-free forward: real tokens only, rows grouped by tenant
            slots = store.slots(list(tenants))
            pb = self.model.pack(input_ids, lengths, slots, token_type_ids)
            with torch.no_grad():
                if head is None:
                    return self.model.encode_pooled_packed(pb, store, pooling)
                h = self.model.encode_packed(pb, store)
                return self.model.heads_packed(h, pb, pooling, **head)
        if store is self.store:
            assembler = self._get_assembler()
        else:  # this batch's staging cache
            kind = IndexSelectBatchAssembler if self._assembler_kind == "index_select" else BatchAssembler
            assembler = kind(store, cfg)
        batch = assembler.batch_lora(list(tenants), input_ids.shape[1], lengths)

        def dev(t):
            if t is None or t.device == cfg.device:
                return t
            return t.pin_memory().to(cfg.device, non_blocking=True) if t.device.type == "cpu" else t.to(cfg.device)

        with torch.no_grad():
            pooled = self.model.encode_pooled(dev(input_ids), dev(attention_mask), batch, dev(token_type_ids),
                                              True, pooling)
            if head is not None:
                head_forward(pooled, pooling="none", **head)
            return pooled

    def _encode(self, texts: Sequence[str], tenants: Sequence[str], text_pairs: Sequence[str] | None = None,
                pooling: str | None = None) -> Tensor:
        """Pooled ``(N, H)`` representations, one row per input, in input order."""
        if len(texts) != len(tenants):
            raise ValueError(
                f"got {len(texts)} texts but {len(tenants)} tenant ids; each text is served by exactly one "
                "tenant's adapter"
            )
        if text_pairs is not None and len(text_pairs) != len(texts):
            raise ValueError(f"got {len(texts)} texts but {len(text_pairs)} pair texts")
        pooling = validate_pooling(pooling or self.pooling)
        cfg = self.config
        if not texts:
            return torch.empty(0, cfg.hidden_size, dtype=cfg.dtype, device=cfg.device)
        pairs = list(text_pairs) if text_pairs is not None else [None] * len(texts)
        items = list(zip(texts, tenants, pairs))
        outputs: list[Tensor] = []
        for chunk, n_valid in chunk_and_pad(items, cfg.batch_size):
            chunk_texts = [c[0] for c in chunk]
            chunk_tenants = [c[1] for c in chunk]
            chunk_pairs = None if text_pairs is None else [c[2] for c in chunk]
            enc = self._tokenize(chunk_texts, chunk_pairs)
            pooled = self.encode_tokens(enc["input_ids"], enc["attention_mask"], chunk_tenants,
                                        enc.get("token_type_ids"), pooling)
            outputs.append(pooled[:n_valid])
        return torch.cat(outputs, dim=0)

    def check_device_status(self) -> None:
        """Raise if a kernel flagged a bad slot/segment or a timeout since the last check."""
        from latefuse_b200 import _native as nat

        status = getattr(getattr(self.model, "_runner", None), "status", None)
        if status is None:
            return
        bits = int(status.item())
        if bits:
            status.zero_()
            raise RuntimeError(f"device status {bits:#x}: {nat.decode_status(bits)}")


class MultiTenantEmbedder(TaskPipeline):
    """Embed texts under many tenants' adapters in one shared forward pass.

    Pooling defaults to ``"cls"`` (``src/latefuse/tasks/embedding.py:39-44``).
    """

    def __init__(self, *args, pooling: str = "cls", **kwargs):
        super().__init__(*args, pooling=pooling, **kwargs)

    @classmethod
    def from_pretrained(cls, model_name: str, *, pooling: str = "cls", **kwargs):
        return super().from_pretrained(model_name, pooling=pooling, **kwargs)

    def embed(self, texts: Sequence[str], tenants: Sequence[str] | str, *, normalize: bool = True,
              pooling: str | None = None) -> Tensor:
        """Embed ``texts``, each under its own tenant's adapter; ``(len(texts), H)``."""
        tenants = self._broadcast_tenants(tenants, len(texts))
        vectors = self._encode(texts, tenants, pooling=pooling)
        if normalize and vectors.numel():
            vectors = l2_normalize(vectors)
        return vectors

    def embed_tokens(self, input_ids: Tensor, attention_mask: Tensor | None, tenants: Sequence[str] | str, *,
                     normalize: bool = True, pooling: str | None = None,
                     token_type_ids: Tensor | None = None) -> Tensor:
        """Embed one pre-tokenized batch (any row count up to the model's limits)."""
        tenants = self._broadcast_tenants(tenants, input_ids.shape[0])
        vectors = self.encode_tokens(input_ids, attention_mask, tenants, token_type_ids, pooling)
        if normalize and vectors.numel():
            vectors = l2_normalize(vectors)
        return vectors

    def embed_tokens_stream(self, batches, *, depth: int = 2, normalize: bool = True,
                            pooling: str | None = None) -> Iterator[Tensor]:
        """:meth:`embed_tokens` over an iterable of ``(input_ids, attention_mask, tenants)``
        host batches with up to ``depth`` in flight (:func:`stream_to_host`): each batch's
        embeddings come back as a pinned host tensor, in order."""
        return stream_to_host(lambda ids, mask, tenants: self.embed_tokens(ids, mask, tenants, normalize=normalize,
                                                                          pooling=pooling), batches, depth)

    @staticmethod
    def _broadcast_tenants(tenants: Sequence[str] | str, n: int) -> list[str]:
        if isinstance(tenants, str):
            return [tenants] * n
        return list(tenants)


class _HeadTask(TaskPipeline):
    def __init__(self, *args, heads: HeadStore | None = None, **kwargs):
        super().__init__(*args, **kwargs)
        self.heads = heads if heads is not None else HeadStore(self.config)

    def _score(self, pooled: Tensor, tenants: list[str]) -> tuple[Tensor, Tensor, list[int]]:
        """(logits (N, n_max) model dtype, probs (N, n_max) f32, num_labels) on the device."""
        table, num_labels, n_max = self.heads.head_table(tenants)
        coef, bias = self.heads.packed
        N = pooled.shape[0]
        logits = torch.empty(N, n_max, dtype=self.config.dtype, device=pooled.device)
        probs = torch.empty(N, n_max, dtype=torch.float32, device=pooled.device)
        head_forward(pooled, pooling="none", coef=coef, bias=bias, head_table=table, n_max=n_max,
                     logits_out=logits, probs_out=probs)
        return logits, probs, num_labels

    def _score_tokens(self, input_ids: Tensor, attention_mask: Tensor | None, tenants: list[str],
                      token_type_ids: Tensor | None = None,
                      n_max: int | None = None) -> tuple[Tensor, Tensor, list[int]]:
        """Encode one pre-tokenized batch and score it with its tenants' heads in the
        same pass: ``(logits (B, n_max), probs (B, n_max), num_labels)`` on the device,
        ``n_max`` at least the widest head of the batch."""
        table, num_labels, widest = self.heads.head_table(tenants)
        n_max = max(widest, n_max or 0)
        coef, bias = self.heads.packed
        B, dev = input_ids.shape[0], self.config.device
        logits = torch.zeros(B, n_max, dtype=self.config.dtype, device=dev)
        probs = torch.zeros(B, n_max, dtype=torch.float32, device=dev)
        self.encode_tokens(input_ids, attention_mask, tenants, token_type_ids,
                           head=dict(coef=coef, bias=bias, head_table=table, n_max=n_max, logits_out=logits,
                                     probs_out=probs))
        return logits, probs, num_labels

    def _scored_texts(self, texts, tenants, text_pairs=None) -> tuple[Tensor, Tensor, list[int]]:
        """Tokenize in fixed-size chunks, encode and score each chunk in one pass."""
        if len(texts) != len(tenants):
            raise ValueError(f"got {len(texts)} texts but {len(tenants)} tenant ids")
        if text_pairs is not None and len(text_pairs) != len(texts):
            raise ValueError(f"got {len(texts)} texts but {len(text_pairs)} pair texts")
        _, num_labels, n_max = self.heads.head_table(list(tenants))  # unknown tenants fail before any forward
        pairs = list(text_pairs) if text_pairs is not None else [None] * len(texts)
        logits, probs = [], []
        for chunk, n_valid in chunk_and_pad(list(zip(texts, tenants, pairs)), self.config.batch_size):
            enc = self._tokenize([c[0] for c in chunk], None if text_pairs is None else [c[2] for c in chunk])
            lo, pr, _ = self._score_tokens(enc["input_ids"], enc["attention_mask"], [c[1] for c in chunk],
                                           enc.get("token_type_ids"), n_max)
            logits.append(lo[:n_valid])
            probs.append(pr[:n_valid])
        return torch.cat(logits), torch.cat(probs), num_labels


class MultiTenantClassifier(_HeadTask):
    """Classify texts under many tenants' adapters and heads in one forward pass."""

    def _scored(self, texts, tenants):
        if len(texts) != len(tenants):
            raise ValueError(f"got {len(texts)} texts but {len(tenants)} tenant ids")
        if not texts:
            return [], [], []
        logits, probs, num_labels = self._scored_texts(texts, list(tenants))
        return logits.tolist(), probs.tolist(), num_labels

    def logits(self, texts: Sequence[str], tenants: Sequence[str]) -> list[list[float]]:
        """Raw per-tenant logits, ragged: row ``i`` has that tenant's label count."""
        logits, _, num_labels = self._scored(texts, tenants)
        return [row[:n] for row, n in zip(logits, num_labels)]

    def predict_proba(self, texts: Sequence[str], tenants: Sequence[str]) -> list[list[float]]:
        """Per-tenant class probabilities, ragged (softmax over own labels; sigmoid if one)."""
        _, probs, num_labels = self._scored(texts, tenants)
        return [row[:n] for row, n in zip(probs, num_labels)]

    def predict(self, texts: Sequence[str], tenants: Sequence[str]) -> list[int]:
        """Highest-scoring label index per text (``logit > 0`` for single-logit heads)."""
        out = []
        for row in self.logits(texts, tenants):
            if len(row) == 1:
                out.append(int(row[0] > 0.0))
            else:
                out.append(max(range(len(row)), key=row.__getitem__))
        return out

    def encode(self, texts: Sequence[str], tenants: Sequence[str]) -> Tensor:
        """Pooled ``(N, H)`` representations, skipping the heads."""
        return self._encode(texts, tenants)

    def classify_tokens(self, input_ids: Tensor, attention_mask: Tensor | None, tenants: Sequence[str],
                        token_type_ids: Tensor | None = None) -> tuple[Tensor, Tensor, list[int]]:
        """Device ``(logits, probs, num_labels)`` for one pre-tokenized batch."""
        return self._score_tokens(input_ids, attention_mask, list(tenants), token_type_ids)


@dataclass(frozen=True)
class RerankResult:
    """One scored document, carrying its position in the original list."""

    index: int
    document: str
    score: float


class MultiTenantReranker(_HeadTask):
    """Score (query, document) pairs under many tenants' adapters at once."""

    def score(self, queries: Sequence[str], documents: Sequence[str], tenants: Sequence[str] | str) -> list[float]:
        """Relevance score (head column 0) for each pair, in input order."""
        if len(queries) != len(documents):
            raise ValueError(
                f"got {len(queries)} queries but {len(documents)} documents; score() takes parallel lists, "
                "one entry per pair"
            )
        if not queries:
            return []
        tenant_ids = [tenants] * len(queries) if isinstance(tenants, str) else list(tenants)
        logits, _, _ = self._scored_texts(list(queries), tenant_ids, text_pairs=list(documents))
        return logits[:, 0].tolist()

    def rerank(self, query: str, documents: Sequence[str], tenant: str, *, top_k: int | None = None) -> list[RerankResult]:
        """Rank ``documents`` against one ``query`` for one tenant, best first."""
        scores = self.score([query] * len(documents), documents, tenant)
        ranked = sorted(
            (RerankResult(index=i, document=doc, score=s) for i, (doc, s) in enumerate(zip(documents, scores))),
            key=lambda r: r.score,
            reverse=True,
        )
        return ranked if top_k is None else ranked[:top_k]
