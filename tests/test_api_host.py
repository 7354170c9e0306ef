"""Host-side behaviour of the Python API that needs no GPU: configuration
validation, registry, strategies (CPU only)."""

import math

import pytest

import sparse_embedding_b200 as se


def test_registry():
    for name in (se.SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, se.SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME,
                 se.SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME):
        assert se.is_partitioner_registered(name)
    assert not se.is_partitioner_registered("non_existent_algo")
    with pytest.raises(Exception) as e:
        se.create_partitioner("non_existent_algo", 4)
    assert "unknown partitioner" in str(e.value).lower()
    with pytest.raises(ValueError, match="num_partitions must be > 0"):
        se.create_partitioner(se.SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, 0)
    with pytest.raises(ValueError, match="num_shards must be > 0"):
        se.ModuloPartitioner(num_shards=0)
    assert isinstance(se.create_partitioner(se.SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME, 4), se.HashPartitioner)


def test_strategy_binding_and_cache():
    s = se.PartitionStrategy(se.SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME)
    assert s.bind(4) is s.bind(4)
    assert s.bind(4).num_shards == 4
    with pytest.raises(TypeError):
        s.bind(True)
    with pytest.raises(ValueError):
        s.bind(0)
    assert se.create_strategy("sparse_embedding.modulo") is se.create_strategy(se.PartitionSpec.modulo())
    assert se.HashPartition(seed=3).parameters == {"seed": "3"}
    with pytest.raises(ValueError, match="unregistered"):
        se.PartitionSpec("nope")
    p = se.ModuloPartitioner(num_shards=3)
    with pytest.raises(ValueError, match="does not match partitioner configured num_shards"):
        p.partition([1, 2], partition_count=4)


@pytest.mark.parametrize("scale", [0.0, -1.0, float("nan"), float("inf")])
def test_gradient_scale_rejected(scale):
    # test_mixed_precision.py:441-455
    with pytest.raises(ValueError, match="gradient_scale"):
        se.EmbeddingStore(se.EmbeddingConfig(dims=[2], value_dtype="float16", optimizer_dtype="float32",
                                             gradient_dtype="float16", gradient_scale=scale, key_dtype="uint64"),
                          optimizer_config=se.Sgd(lr=0.01))


def test_config_errors():
    with pytest.raises(ValueError, match="optimizer_config cannot be provided"):
        se.EmbeddingStore(se.EmbeddingConfig(dims=[4], enable_optimizer=False), optimizer_config=se.Sgd())
    with pytest.raises(ValueError, match="unsupported dtype"):
        se.EmbeddingStore(se.EmbeddingConfig(dims=[4], value_dtype="float64"))
    with pytest.raises(ValueError, match="unsupported key dtype"):
        se.EmbeddingStore(se.EmbeddingConfig(dims=[4], key_dtype="int8"))
    with pytest.raises(ValueError, match="dims must not be empty"):
        se.EmbeddingStore(se.EmbeddingConfig(dims=[]))
    cfg = se.EmbeddingConfig(dims=[4], value_dtype=float, key_dtype=int)
    assert cfg.value_dtype == "float32" and cfg.key_dtype == "int64"
    assert math.isclose(se.Adagrad().initial_accumulator_value, 0.1)


@pytest.mark.parametrize(
    "factory",
    [
        lambda: se.CustomLutLrPolicy(lut=[]),
        lambda: se.CustomLutLrPolicy(lut=[-0.1]),
        lambda: se.CustomLutLrPolicy(lut=[math.nan]),
        lambda: se.CosineFrequencyLrPolicy(min_lr_ratio=-0.1),
        lambda: se.CosineFrequencyLrPolicy(min_lr_ratio=1.1),
        lambda: se.CosineFrequencyLrPolicy(min_lr_ratio=math.nan),
        lambda: se.CosineFrequencyLrPolicy(max_score=0),
    ],
)
def test_invalid_lr_policy_configuration_is_rejected(factory):
    """tests/test_dynamic_lr.py:117-131."""
    with pytest.raises(ValueError):
        factory()
