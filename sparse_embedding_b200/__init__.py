"""B200-native drop-in for the sparse_embedding hot path.

`EmbeddingStore`, `EmbeddingConfig`, the optimizers, initializers and the
partitioner registry keep the reference's names and behaviour
(sparse_embedding/__init__.py); the work runs in sm_100a kernels behind the C
ABI of libse_gpu.so (include/se_gpu.h).
"""

from .partitioner import (
    SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME,
    SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME,
    SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME,
    SUPPORTED_KEY_DTYPES,
    FastRangePartition,
    FastRangePartitioner,
    HashPartition,
    HashPartitioner,
    ModuloPartition,
    ModuloPartitioner,
    Partitioner,
    PartitionSpec,
    PartitionStrategy,
    create_partitioner,
    create_strategy,
    filter_partition,
    generate_reference_vectors,
    is_partitioner_registered,
    partition,
    register_partitioner,
)
from .unique import async_unique, unique
from .store import (
    Adagrad,
    Adam,
    AutoStorage,
    ConstantLrPolicy,
    CosineFrequencyLrPolicy,
    CustomLutLrPolicy,
    InverseDecayLrPolicy,
    LogDecayLrPolicy,
    LrPolicy,
    SqrtDecayLrPolicy,
    EmbeddingConfig,
    EmbeddingStore,
    Initializer,
    MemoryOnly,
    Optimizer,
    Sgd,
    StorageTuningOptions,
    Uniform,
    Zeros,
)

__version__ = "0.1.0"

__all__ = [
    "Adagrad", "Adam", "AutoStorage", "EmbeddingConfig", "EmbeddingStore", "FastRangePartition",
    "FastRangePartitioner", "HashPartition", "HashPartitioner", "Initializer", "MemoryOnly",
    "ModuloPartition", "ModuloPartitioner", "Optimizer", "PartitionSpec", "PartitionStrategy",
    "Partitioner", "SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME", "SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME",
    "SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME", "SUPPORTED_KEY_DTYPES", "Sgd", "StorageTuningOptions",
    "Uniform", "Zeros", "create_partitioner", "create_strategy", "filter_partition",
    "generate_reference_vectors", "is_partitioner_registered", "partition", "register_partitioner",
]
