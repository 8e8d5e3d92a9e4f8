"""Per-tenant classification heads in one packed device cache.

Mirror of ``src/latefuse/tasks/heads.py`` (``LRHead``, ``HeadStore``).  Every
head's ``coef`` rows and ``intercept`` entries live in two packed buffers
(``(rows, H)`` and ``(rows,)``); a tenant is an ``(offset, num_labels)`` range.
The head kernel gathers each batch row's own range directly, so the reference's
per-batch zero-padded ``(B, max_labels, H)`` copy (``HeadStore.assemble``,
``src/latefuse/tasks/heads.py:125-158``) is not needed on the serving path;
:meth:`HeadStore.assemble` still builds it for API compatibility.
"""

from __future__ import annotations

import torch
from torch import Tensor

from latefuse_b200.batch import BatchedLRWeights
from latefuse_b200.config import LoraServingConfig


class LRHead:
    """One tenant's logistic-regression head: ``coef (num_labels, H)``, ``intercept (num_labels,)``.

    For a head held by a :class:`HeadStore` both are views of the packed cache.
    """

    __slots__ = ("coef", "intercept")

    def __init__(self, coef: Tensor, intercept: Tensor):
        self.coef = coef
        self.intercept = intercept

    @property
    def num_labels(self) -> int:
        return self.coef.shape[0]


class HeadStore:
    """Pre-loaded per-tenant heads, keyed by the same tenant id as the adapter."""

    def __init__(self, config: LoraServingConfig, capacity_rows: int = 1024):
        self._config = config
        self._heads: dict[str, LRHead] = {}
        self._range: dict[str, tuple[int, int]] = {}
        self._free: dict[int, list[int]] = {}
        self._top = 0
        H = config.hidden_size
        self._coef = torch.zeros(max(1, capacity_rows), H, dtype=config.dtype, device=config.device)
        self._bias = torch.zeros(max(1, capacity_rows), dtype=config.dtype, device=config.device)

    # -- packed storage ------------------------------------------------------
    def _grow(self, rows: int) -> None:
        cap = self._coef.shape[0]
        if rows <= cap:
            return
        new_cap = max(rows, cap * 2)
        coef = torch.zeros(new_cap, self._coef.shape[1], dtype=self._coef.dtype, device=self._coef.device)
        bias = torch.zeros(new_cap, dtype=self._bias.dtype, device=self._bias.device)
        coef[:cap].copy_(self._coef)
        bias[:cap].copy_(self._bias)
        self._coef, self._bias = coef, bias
        for tid, (off, n) in self._range.items():  # re-point every head at the new buffers
            self._heads[tid].coef = self._coef[off : off + n]
            self._heads[tid].intercept = self._bias[off : off + n]

    def _alloc(self, n: int) -> int:
        bucket = self._free.get(n)
        if bucket:
            return bucket.pop()
        off = self._top
        self._grow(off + n)
        self._top = off + n
        return off

    def _release(self, tenant_id: str) -> None:
        off, n = self._range.pop(tenant_id)
        self._free.setdefault(n, []).append(off)
        del self._heads[tenant_id]

    # -- reference API -------------------------------------------------------
    def _checked(self, tenant_id: str, coef, intercept) -> tuple[Tensor, Tensor]:
        """``coef`` as ``(n, H)`` and ``intercept`` as ``(n,)`` in the serving dtype, or a
        ``ValueError`` whose wording the reference's callers match on
        (``src/latefuse/tasks/heads.py:58-96``)."""
        cfg = self._config
        c = torch.as_tensor(coef, dtype=cfg.dtype, device=cfg.device)
        b = torch.as_tensor(intercept, dtype=cfg.dtype, device=cfg.device)
        c = c.reshape(1, -1) if c.dim() == 1 else c
        b = b.reshape(1) if b.dim() == 0 else b
        if c.dim() != 2:
            raise ValueError(f"coef for '{tenant_id}' must be (num_labels, H) or (H,), got {tuple(c.shape)}")
        n, width = c.shape
        if width != cfg.hidden_size:
            raise ValueError(
                f"coef for '{tenant_id}' has hidden size {width}, but {cfg.model_name} pools to "
                f"{cfg.hidden_size}. A head fitted on a different backbone cannot be served by this one."
            )
        if tuple(b.shape) != (n,):
            raise ValueError(f"intercept for '{tenant_id}' has shape {tuple(b.shape)}, expected {(n,)} to match coef")
        return c, b

    def load(self, tenant_id: str, coef, intercept) -> None:
        """Store ``tenant_id``'s head in the packed cache, replacing any earlier one.

        ``coef`` is ``(num_labels, H)``; a 1-D ``(H,)`` vector is a one-logit head
        (binary, or a reranker's score) and then ``intercept`` may be a scalar.
        Anything array-like is accepted and cast to the serving dtype.

        Raises:
            ValueError: ``coef`` is not 1-D or 2-D, its width is not the encoder's
                        hidden size, or ``intercept`` has a different label count.
        """
        coef_t, intercept_t = self._checked(tenant_id, coef, intercept)
        n = coef_t.shape[0]
        if tenant_id in self._range:
            self._release(tenant_id)
        off = self._alloc(n)
        self._coef[off : off + n].copy_(coef_t)
        self._bias[off : off + n].copy_(intercept_t)
        self._range[tenant_id] = (off, n)
        self._heads[tenant_id] = LRHead(self._coef[off : off + n], self._bias[off : off + n])

    def load_from_sklearn(self, tenant_id: str, classifier) -> None:
        """Cache a head from a fitted scikit-learn linear classifier (``coef_`` / ``intercept_``)."""
        for attr in ("coef_", "intercept_"):
            if not hasattr(classifier, attr):
                raise ValueError(
                    f"{type(classifier).__name__} has no '{attr}'; expected a fitted linear classifier "
                    "(e.g. sklearn LogisticRegression)"
                )
        self.load(tenant_id, classifier.coef_, classifier.intercept_)

    def load_from_file(self, tenant_id: str, path: str) -> None:
        """Cache a head from a torch file holding ``{"coef": ..., "intercept": ...}``."""
        state = torch.load(path, map_location=self._config.device, weights_only=True)
        missing = {"coef", "intercept"} - set(state)
        if missing:
            raise KeyError(f"{path} is missing {sorted(missing)}; expected a dict with 'coef' and 'intercept'")
        self.load(tenant_id, state["coef"], state["intercept"])

    def assemble(self, tenant_ids: list[str]) -> BatchedLRWeights:
        """One batch of heads zero-padded to the widest present (reference layout)."""
        heads = [self.get(t) for t in tenant_ids]
        num_labels = [h.num_labels for h in heads]
        max_labels = max(num_labels)
        cfg = self._config
        coef = torch.zeros(len(heads), max_labels, cfg.hidden_size, dtype=cfg.dtype, device=cfg.device)
        intercept = torch.zeros(len(heads), max_labels, dtype=cfg.dtype, device=cfg.device)
        for i, head in enumerate(heads):
            coef[i, : head.num_labels] = head.coef
            intercept[i, : head.num_labels] = head.intercept
        batched = BatchedLRWeights()
        batched.coef = coef
        batched.intercept = intercept
        batched.num_labels = num_labels
        return batched

    def head_table(self, tenant_ids: list[str]) -> tuple[Tensor, list[int], int]:
        """Kernel view of one batch: a device int32 ``(2, B)`` table of (offset, num_labels)
        rows into the packed cache, the label counts, and their maximum."""
        ranges = [self._range_of(t) for t in tenant_ids]
        num_labels = [n for _, n in ranges]
        table = torch.tensor([[o for o, _ in ranges], num_labels], dtype=torch.int32)
        if self._coef.device.type == "cuda":
            table = table.pin_memory().to(self._coef.device, non_blocking=True)
        return table, num_labels, max(num_labels) if num_labels else 0

    def _range_of(self, tenant_id: str) -> tuple[int, int]:
        if tenant_id not in self._range:
            raise KeyError(
                f"No head for tenant '{tenant_id}'. Call load(), load_from_sklearn() or load_from_file() first."
            )
        return self._range[tenant_id]

    @property
    def packed(self) -> tuple[Tensor, Tensor]:
        """The packed ``(rows, H)`` coef and ``(rows,)`` intercept buffers."""
        return self._coef, self._bias

    def get(self, tenant_id: str) -> LRHead:
        self._range_of(tenant_id)
        return self._heads[tenant_id]

    def evict(self, tenant_id: str) -> None:
        if tenant_id not in self._range:
            raise KeyError(f"Head for tenant '{tenant_id}' is not resident.")
        self._release(tenant_id)

    def tenant_ids(self) -> list[str]:
        return list(self._range)

    def num_labels(self, tenant_id: str) -> int:
        return self.get(tenant_id).num_labels

    def __contains__(self, tenant_id: object) -> bool:
        return tenant_id in self._range

    def __len__(self) -> int:
        return len(self._range)

    def memory_bytes(self) -> int:
        """Bytes held by resident heads (coef rows + intercepts)."""
        e = self._coef.element_size()
        return sum(n * (self._config.hidden_size + 1) * e for _, n in self._range.values())
