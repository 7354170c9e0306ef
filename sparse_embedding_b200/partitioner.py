"""Partitioners: the registry, the three registered algorithms and the elastic
strategy objects, with the reference's names and behaviour
(sparse_embedding/src/ops/partitioner_registry.cpp:24-83,
sparse_embedding/src/bindings/module.cpp:195-330, 1080-1168,
sparse_embedding/partitioner.py:36-232). Partition ids are computed by the
sm_100a kernels of libse_gpu.so (se_partition / se_filter).
"""

from __future__ import annotations

import asyncio
import threading
from collections.abc import Mapping
from typing import Any, Callable

import numpy as np

from . import _native as N
from ._tensors import as_input, data_ptr, empty_like_space

SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME = "sparse_embedding.modulo"
SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME = "sparse_embedding.hash"
SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME = "sparse_embedding.fast_range"
SUPPORTED_KEY_DTYPES = frozenset({"int32", "uint32", "int64", "uint64"})

_DEFAULT_DEVICE = None


def _device_for(arr) -> int:
    if arr.cuda_device is not None:
        return arr.cuda_device
    global _DEFAULT_DEVICE
    if _DEFAULT_DEVICE is None:
        from ._tensors import torch_mod

        torch = torch_mod()
        if not torch.cuda.is_available():
            raise RuntimeError("partitioning runs on the GPU and needs a CUDA device")
        _DEFAULT_DEVICE = torch.cuda.current_device()
    return _DEFAULT_DEVICE


class Partitioner:
    """PyPartitioner (bindings/module.cpp:195-330)."""

    _kind = "modulo"

    def __init__(self, num_shards: int):
        if int(num_shards) <= 0:
            raise ValueError("num_shards must be > 0")
        if int(num_shards) > 0xFFFFFFFF:
            raise OverflowError("num_shards must fit in uint32")
        self.num_shards = int(num_shards)

    @property
    def name(self) -> str:
        return {"modulo": SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME,
                "hash": SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME,
                "fast_range": SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME}[self._kind]

    def _check_count(self, partition_count):
        if partition_count is not None and int(partition_count) != self.num_shards:
            raise ValueError(
                f"partition_count ({int(partition_count)}) does not match partitioner "
                f"configured num_shards ({self.num_shards})")

    def _keys(self, keys):
        k = as_input(keys, "keys")
        if k.dtype not in N.KEY_CODES:
            raise ValueError(f"unsupported key dtype: {k.dtype}")
        return k

    def partition(self, keys, partition_count: int | None = None, domain_size: int | None = None,
                  num_threads: int = 0):
        """Partition id (uint32) of every key."""
        del domain_size, num_threads
        self._check_count(partition_count)
        k = self._keys(keys)
        out = empty_like_space(k, (k.size,), "uint32")
        if k.size:
            N.check(N.lib().se_partition(N.PART_CODES[self._kind], self.num_shards, N.KEY_CODES[k.dtype],
                                         k.ptr, k.size, data_ptr(out), _device_for(k), k.stream))
        return out

    def filter(self, keys, target_shard: int, partition_count: int | None = None,
               domain_size: int | None = None, num_threads: int = 0):
        """Boolean mask: partition id of each key == target_shard."""
        del domain_size, num_threads
        self._check_count(partition_count)
        k = self._keys(keys)
        out = empty_like_space(k, (k.size,), "bool")
        if k.size:
            N.check(N.lib().se_filter(N.PART_CODES[self._kind], self.num_shards, N.KEY_CODES[k.dtype],
                                      k.ptr, k.size, int(target_shard), data_ptr(out), _device_for(k),
                                      k.stream))
        return out

    async def async_partition(self, keys, partition_count: int | None = None,
                              domain_size: int | None = None, num_threads: int = 0):
        return await asyncio.to_thread(self.partition, keys, partition_count, domain_size, num_threads)

    async def async_filter(self, keys, target_shard: int, partition_count: int | None = None,
                           domain_size: int | None = None, num_threads: int = 0):
        return await asyncio.to_thread(self.filter, keys, target_shard, partition_count, domain_size,
                                       num_threads)

    def route(self, keys):
        """Groups CUDA keys by partition, stably (exchange step of the sharded
        store): returns (send_keys, send_positions, counts)."""
        from ._tensors import torch_mod

        torch = torch_mod()
        k = self._keys(keys)
        if k.cuda_device is None:
            raise ValueError("route takes CUDA tensors")
        dev = f"cuda:{k.cuda_device}"
        send_keys = torch.empty_like(keys)
        send_pos = torch.empty(k.size, dtype=torch.int32, device=dev)
        counts = torch.empty(self.num_shards, dtype=torch.int32, device=dev)
        N.check(N.lib().se_partition_route(N.PART_CODES[self._kind], self.num_shards, N.KEY_CODES[k.dtype],
                                           k.ptr, k.size, send_keys.data_ptr(), send_pos.data_ptr(),
                                           counts.data_ptr(), k.cuda_device, k.stream))
        return send_keys, send_pos, counts


class ModuloPartitioner(Partitioner):
    """ModuloPartitioner (ops/partitioner.hpp:72-179): signed floor modulo."""

    _kind = "modulo"


class HashPartitioner(Partitioner):
    """HashPartitioner (ops/partitioner.hpp:222-406): splitmix64 / murmur fmix32."""

    _kind = "hash"


class FastRangePartitioner(Partitioner):
    """FastRangePartitioner (ops/partitioner.hpp:181-220): Lemire fast range."""

    _kind = "fast_range"


# ---------------------------------------------------------------------------
# Registry (PartitionerRegistry, ops/partitioner_registry.cpp:24-83)
# ---------------------------------------------------------------------------

_registry_lock = threading.Lock()
_factories: dict[str, Callable[[int, Mapping[str, str]], Partitioner]] = {
    SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME: lambda n, p: ModuloPartitioner(n),
    SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME: lambda n, p: HashPartitioner(n),
    SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME: lambda n, p: FastRangePartitioner(n),
}


def register_partitioner(name: str, factory: Callable[[int, Mapping[str, str]], Partitioner]) -> None:
    if factory is None:
        raise ValueError("partitioner factory cannot be empty")
    with _registry_lock:
        _factories[str(name)] = factory


def is_partitioner_registered(name: str) -> bool:
    with _registry_lock:
        return name in _factories


def create_partitioner(name: str, num_partitions: int, parameters: Mapping[str, Any] | None = None) -> Partitioner:
    if int(num_partitions) <= 0:
        raise ValueError("num_partitions must be > 0")
    with _registry_lock:
        f = _factories.get(name)
    if f is None:
        raise ValueError(f"unknown partitioner: {name}")
    params = {str(k): str(v) for k, v in (parameters or {}).items()}
    return f(int(num_partitions), params)


# ---------------------------------------------------------------------------
# PartitionSpec and strategies (checkpoint/base.py:382-470; partitioner.py:36-232)
# ---------------------------------------------------------------------------


class PartitionSpec:
    """Declarative partition specification (name + parameters)."""

    __slots__ = ("_name", "_parameters")

    def __init__(self, name: str, parameters: Mapping[str, object] | None = None):
        if not isinstance(name, str):
            raise TypeError("partition spec name must be a string")
        if not name.strip():
            raise ValueError("partition spec name must be non-empty")
        if len(name.encode("utf-8")) > 128:
            raise ValueError("partition spec name is too long")
        params = parameters if parameters is not None else {}
        if not isinstance(params, Mapping):
            raise TypeError("partition spec parameters must be a mapping")
        if not is_partitioner_registered(name):
            raise ValueError(f"unregistered partition algorithm: {name!r}")
        self._name = name
        self._parameters = dict(params)

    @property
    def name(self) -> str:
        return self._name

    @property
    def parameters(self) -> Mapping[str, object]:
        return dict(self._parameters)

    def __eq__(self, other):
        return isinstance(other, PartitionSpec) and (self._name, self._parameters) == (other._name, other._parameters)

    def __hash__(self):
        return hash((self._name, tuple(sorted((str(k), str(v)) for k, v in self._parameters.items()))))

    def __repr__(self):
        return f"PartitionSpec(name={self._name!r}, parameters={dict(self._parameters)!r})"

    @classmethod
    def modulo(cls) -> "PartitionSpec":
        return cls(SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, {})

    @classmethod
    def hash(cls, *, seed: int | None = None) -> "PartitionSpec":
        return cls(SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME, {} if seed is None else {"seed": str(seed)})

    @classmethod
    def fast_range(cls) -> "PartitionSpec":
        return cls(SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME, {})


class PartitionStrategy:
    """Late-binding partition strategy with a per-count partitioner cache."""

    __slots__ = ("_spec", "_kernel_cache", "_lock")

    def __init__(self, name: str = SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME,
                 parameters: Mapping[str, object] | None = None):
        self._spec = PartitionSpec(name, parameters)
        self._kernel_cache: dict[int, Partitioner] = {}
        self._lock = threading.Lock()

    @property
    def name(self) -> str:
        return self._spec.name

    @property
    def parameters(self) -> Mapping[str, object]:
        return self._spec.parameters

    @property
    def spec(self) -> PartitionSpec:
        return self._spec

    def bind(self, partition_count: int) -> Partitioner:
        if not isinstance(partition_count, int) or isinstance(partition_count, bool):
            raise TypeError("partition_count must be an integer")
        if partition_count <= 0:
            raise ValueError(f"partition_count must be positive; got {partition_count}")
        with self._lock:
            kernel = self._kernel_cache.get(partition_count)
            if kernel is None:
                kernel = create_partitioner(self.name, partition_count, dict(self.parameters))
                self._kernel_cache[partition_count] = kernel
            return kernel

    def __call__(self, values, *, partition_count: int, domain_size: int | None = None,
                 num_threads: int = 0, **kwargs):
        return self.bind(partition_count).partition(values, partition_count=partition_count,
                                                    num_threads=num_threads)

    def filter(self, values, target_shard: int, *, partition_count: int, domain_size: int | None = None,
               num_threads: int = 0, **kwargs):
        return self.bind(partition_count).filter(values, target_shard=target_shard,
                                                 partition_count=partition_count, num_threads=num_threads)

    def __repr__(self):
        return f"PartitionStrategy(name={self.name!r}, parameters={dict(self.parameters)!r})"


class ModuloPartition(PartitionStrategy):
    def __init__(self, parameters: Mapping[str, object] | None = None):
        super().__init__(SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, parameters)


class HashPartition(PartitionStrategy):
    def __init__(self, parameters: Mapping[str, object] | None = None, *, seed: int | None = None):
        params = dict(parameters or {})
        if seed is not None:
            params["seed"] = str(seed)
        super().__init__(SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME, params)


class FastRangePartition(PartitionStrategy):
    def __init__(self, parameters: Mapping[str, object] | None = None):
        super().__init__(SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME, parameters)


_STRATEGY_CACHE: dict = {}
_STRATEGY_LOCK = threading.Lock()


def _strategy(algorithm: str, parameters: Mapping[str, object] | None) -> PartitionStrategy:
    key = (algorithm, tuple(sorted((str(k), str(v)) for k, v in (parameters or {}).items())))
    with _STRATEGY_LOCK:
        s = _STRATEGY_CACHE.get(key)
        if s is None:
            s = PartitionStrategy(algorithm, parameters)
            _STRATEGY_CACHE[key] = s
        return s


def partition(keys, *, partition_count: int, domain_size: int | None = None,
              algorithm: str = SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, num_threads: int = 0, **parameters):
    return _strategy(algorithm, parameters)(keys, partition_count=partition_count, domain_size=domain_size,
                                            num_threads=num_threads)


def filter_partition(keys, target_shard: int, *, partition_count: int, domain_size: int | None = None,
                     algorithm: str = SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, num_threads: int = 0,
                     **parameters):
    return _strategy(algorithm, parameters).filter(keys, target_shard, partition_count=partition_count,
                                                   domain_size=domain_size, num_threads=num_threads)


def create_strategy(spec_or_name: PartitionSpec | str = SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME,
                    parameters: Mapping[str, object] | None = None) -> PartitionStrategy:
    if isinstance(spec_or_name, PartitionSpec):
        return _strategy(spec_or_name.name, spec_or_name.parameters)
    if isinstance(spec_or_name, str):
        return _strategy(spec_or_name, parameters)
    raise TypeError("spec_or_name must be a PartitionSpec or string algorithm name; got "
                    f"{type(spec_or_name).__name__}")


def generate_reference_vectors(assignment_name: str, key_dtype: str, partition_count: int,
                               parameters: Mapping[str, object] | None = None, *,
                               sample_keys=None) -> tuple[np.ndarray, np.ndarray]:
    """Keys and their partition ids (checkpoint/reference_vectors.py:12-67): the
    default key sets are the reference's boundary keys for each dtype."""
    if partition_count <= 0:
        raise ValueError("partition_count must be > 0")
    np_dtype = np.dtype(key_dtype)
    if sample_keys is None:
        if np.issubdtype(np_dtype, np.signedinteger):
            keys_list = [-(1 << 30), -1048576, -1024, -3, -2, -1, 0, 1, 2, 3, 1024, 1048576, (1 << 30) - 1]
        else:
            keys_list = [0, 1, 2, 3, 1024, 1048576, (1 << 30) - 1, (1 << 31) - 1]
        keys_arr = np.array(keys_list, dtype=np_dtype)
    else:
        keys_arr = np.array(sample_keys, dtype=np_dtype)
    p = create_partitioner(assignment_name, partition_count, parameters)
    ranks = np.asarray(p.partition(keys_arr), dtype=np.uint32)
    return keys_arr, ranks
