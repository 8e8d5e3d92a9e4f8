"""Seeded synthetic serving inputs (mirror of ``src/latefuse/benchmark/synthetic.py``),
plus the workload generators of the serving benchmarks: Zipf tenant streams
(``src/latefuse/benchmark/run.py:170-174``) and ragged padded batches."""

from __future__ import annotations

import numpy as np
import torch

from latefuse_b200.config import LoraServingConfig
from latefuse_b200.store import AdapterStore


def make_synthetic_adapters(store: AdapterStore, n: int, seed: int = 42) -> None:
    """Register ``adapter_0 .. adapter_{n-1}`` with ``load_synthetic(seed + i)``."""
    for i in range(n):
        store.load_synthetic(f"adapter_{i}", seed=seed + i)


def make_synthetic_inputs(config: LoraServingConfig, batch_size: int) -> dict:
    """Token ids uniform in [1, 30000) and an all-ones mask, ``(batch_size, max_seq_len)``."""
    return {
        "input_ids": torch.randint(low=1, high=30000, size=(batch_size, config.max_seq_len), device=config.device),
        "attention_mask": torch.ones(batch_size, config.max_seq_len, dtype=torch.long, device=config.device),
    }


def make_synthetic_lr_weights(config: LoraServingConfig, num_labels: int = 10) -> tuple:
    """Random head: coef ``(1, num_labels, H)`` ~ N(0,1), zero intercept."""
    coef = torch.randn(1, num_labels, config.hidden_size, dtype=config.dtype, device=config.device)
    intercept = torch.zeros(1, num_labels, dtype=config.dtype, device=config.device)
    return coef, intercept


def zipf_probabilities(n_population: int, alpha: float = 1.1) -> np.ndarray:
    ranks = np.arange(1, n_population + 1, dtype=np.float64)
    p = 1.0 / np.power(ranks, alpha)
    return p / p.sum()


def zipf_tenants(n_population: int, n_rows: int, alpha: float = 1.1, seed: int = 0) -> np.ndarray:
    """Tenant indices of ``n_rows`` requests drawn Zipf(alpha) over ``n_population``."""
    rng = np.random.default_rng(seed)
    return rng.choice(n_population, size=n_rows, p=zipf_probabilities(n_population, alpha))


def ragged_batch(batch: int, seq: int, *, min_len: int, max_len: int, vocab: int, pad_id: int = 1,
                 cls_id: int = 0, low_id: int = 5, seed: int = 0,
                 stratified: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Host ``(input_ids, attention_mask)`` of ``batch`` right-padded rows with lengths
    uniform in ``[min_len, max_len]``: CLS at position 0, ids uniform in ``[low_id, vocab)``
    elsewhere in the real part, ``pad_id`` with mask 0 after it.

    With ``stratified`` the lengths are a Latin-hypercube draw: row ``i`` of a random
    permutation takes one uniform draw from the ``i``-th of ``batch`` equal bands of
    ``[min_len, max_len + 1)``.  Each length is still uniform over the range, and the
    batch's total is within one band of its expectation, so batches of one seed and
    different sizes carry the same work per row."""
    g = torch.Generator().manual_seed(seed)
    if stratified:
        band = (max_len + 1 - min_len) / batch
        u = torch.rand(batch, generator=g, dtype=torch.float64)
        perm = torch.randperm(batch, generator=g).to(torch.float64)
        lengths = (min_len + (perm + u) * band).floor().clamp(max=max_len).to(torch.int64)
    else:
        lengths = torch.randint(min_len, max_len + 1, (batch,), generator=g)
    ids = torch.randint(low_id, vocab, (batch, seq), generator=g)
    pos = torch.arange(seq).unsqueeze(0)
    mask = (pos < lengths.unsqueeze(1)).to(torch.int64)
    ids = torch.where(mask.bool(), ids, torch.full_like(ids, pad_id))
    ids[:, 0] = cls_id
    return ids, mask
