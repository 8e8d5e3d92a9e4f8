"""Oracle for the task-level glue (CPU).

``chunk_and_pad`` restates ``src/latefuse/tasks/batching.py:23-52``; ``embed``
restates ``TaskPipeline._encode`` + ``MultiTenantEmbedder.embed``
(``src/latefuse/tasks/base.py:228-279``, ``src/latefuse/tasks/embedding.py:46-71``)
over a :class:`oracle.encoder.HookedEncoder`.
"""

from __future__ import annotations

import torch

from oracle.head import normalize


def chunk_and_pad(items, batch_size: int):
    if batch_size <= 0:
        raise ValueError(f"batch_size must be positive, got {batch_size}")
    for start in range(0, len(items), batch_size):
        chunk = list(items[start : start + batch_size])
        n_valid = len(chunk)
        if n_valid < batch_size:
            chunk.extend([chunk[-1]] * (batch_size - n_valid))
        yield chunk, n_valid


@torch.no_grad()
def embed(encoder, tokenizer, texts, tenants, *, batch_size: int, max_seq_len: int, pooling: str = "cls",
          do_normalize: bool = True, text_pairs=None):
    """Chunk/pad, tokenize with ``padding="max_length"``, encode, slice, normalise."""
    pairs = list(text_pairs) if text_pairs is not None else [None] * len(texts)
    outs = []
    for chunk, n_valid in chunk_and_pad(list(zip(texts, tenants, pairs)), batch_size):
        args = ([c[0] for c in chunk],) if text_pairs is None else ([c[0] for c in chunk], [c[2] for c in chunk])
        enc = tokenizer(*args, padding="max_length", truncation=True, max_length=max_seq_len, return_tensors="pt")
        pooled = encoder.encode_pooled(enc["input_ids"], enc["attention_mask"], [c[1] for c in chunk], pooling,
                                       token_type_ids=enc.get("token_type_ids"))
        outs.append(pooled[:n_valid])
    out = torch.cat(outs, 0)
    return normalize(out) if do_normalize else out
