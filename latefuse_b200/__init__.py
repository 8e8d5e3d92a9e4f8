"""LateFuse-B200: multi-tenant late-fusion LoRA serving for encoder models on NVIDIA B200.

Many LoRA-adapted encoders are served in one shared forward pass: the frozen
base projections run once over a mixed-tenant batch; each row gets its own
low-rank delta ``B_t (A_t x)`` and each tenant's classification head is applied
to its pooled output.  The API is LateFuse's (``MultiTenantEmbedder``,
``MultiTenantClassifier``, ``MultiTenantReranker``, ``register_adapter`` /
``register_synthetic`` / ``evict_adapter``, ``heads.load`` ...); underneath, the
per-row deltas, pooling, normalisation and heads run in hand-written sm_100a
kernels (``liblatefuse_b200.so``, C ABI in ``include/latefuse_b200.h``) that read
adapters in place from one slot-indexed device cache.

    from latefuse_b200 import MultiTenantEmbedder

    embedder = MultiTenantEmbedder.from_pretrained("BAAI/bge-m3", dtype=torch.bfloat16)
    embedder.register_adapter("acme", "adapters/acme")
    vectors = embedder.embed(["renew my policy"], ["acme"])
"""

from latefuse_b200.batch import (
    BatchAssembler,
    BatchedLRWeights,
    BatchLora,
    IndexSelectBatchAssembler,
    LayerwiseBatchedWeights,
)
from latefuse_b200.config import LoraServingConfig
from latefuse_b200.engine import EncoderWithLora, HFEncoderWithLora
from latefuse_b200.head import POOLING_STRATEGIES, LRHeadOps, pool_tokens, validate_pooling
from latefuse_b200.heads import HeadStore, LRHead
from latefuse_b200.loaders import load_peft_adapter, peft_key_fn
from latefuse_b200.lora import LoraOps, SegmentTable, lora_apply
from latefuse_b200.rank_buckets import RankBucketStore
from latefuse_b200.store import AdapterStore, LoraWeight
from latefuse_b200.tasks import (
    ASSEMBLERS,
    ENGINES,
    MultiTenantClassifier,
    MultiTenantEmbedder,
    MultiTenantReranker,
    RerankResult,
    TaskPipeline,
    chunk_and_pad,
)

__version__ = "0.1.0"

__all__ = [
    # Task-level API.
    "MultiTenantEmbedder",
    "MultiTenantClassifier",
    "MultiTenantReranker",
    "RerankResult",
    "TaskPipeline",
    "ENGINES",
    "ASSEMBLERS",
    "chunk_and_pad",
    # Configuration and adapter loading.
    "LoraServingConfig",
    "load_peft_adapter",
    "peft_key_fn",
    "POOLING_STRATEGIES",
    "validate_pooling",
    "pool_tokens",
    # Stores.
    "AdapterStore",
    "RankBucketStore",
    "LoraWeight",
    "HeadStore",
    "LRHead",
    # Engines.
    "EncoderWithLora",
    "HFEncoderWithLora",
    # Batch assembly and the low-level ops.
    "BatchAssembler",
    "IndexSelectBatchAssembler",
    "BatchedLRWeights",
    "LayerwiseBatchedWeights",
    "BatchLora",
    "SegmentTable",
    "LoraOps",
    "LRHeadOps",
    "lora_apply",
    "__version__",
]
