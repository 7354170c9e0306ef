"""Python surface of the GPU store, mirroring the reference's `_core` module.

Names, arguments, defaults and error classes follow the reference's nanobind
bindings (sparse_embedding/src/bindings/module.cpp:383-724) and its Python
package (sparse_embedding/__init__.py:63-135), so code written against the
reference's `EmbeddingStore` runs unchanged; every operation goes through the
C ABI of libse_gpu.so (include/se_gpu.h) to the sm_100a kernels.
"""

from __future__ import annotations

import ctypes as C
import math
import os
from typing import Any, Sequence

import numpy as np

from . import _native as N
from ._tensors import Arr, as_input, data_ptr, empty_like_space

# ---------------------------------------------------------------------------
# Configuration objects
# ---------------------------------------------------------------------------


def _parse_value_dtype(name: str, label: str) -> str:
    # se::parse_value_dtype (sparse_embedding/src/common/dtypes.hpp:157-167)
    aliases = {"float32": "float32", "f32": "float32", "float16": "float16", "f16": "float16",
               "bfloat16": "bfloat16", "bf16": "bfloat16"}
    if name not in aliases:
        raise ValueError(f"unsupported {label}: {name}")
    return aliases[name]


def _parse_key_dtype(name: str) -> str:
    # se::parse_key_dtype (dtypes.hpp:68-78)
    if name not in N.KEY_CODES:
        raise ValueError(f"unsupported key dtype: {name}")
    return name


def _to_str(dt: Any) -> str:
    # sparse_embedding/__init__.py:87-102
    if dt is None:
        return ""
    if hasattr(dt, "__name__"):
        name = dt.__name__
    elif hasattr(dt, "name"):
        name = dt.name
    else:
        name = str(dt)
    name = name.replace("torch.", "")
    if name == "float":
        return "float32"
    if name == "int":
        return "int64"
    return name


class StorageTuningOptions:
    """Accepted for API compatibility (storage_topology.hpp:19-27).

    Host paging is out of scope for the GPU store: the table lives in HBM.
    target_capacity_keys, when set, sizes each table's initial capacity.
    """

    def __init__(self, target_capacity_keys: int = 0, memory_budget_bytes: int = 0,
                 entries_per_page: int = 0, max_pages: int = 0, workload: Any = None,
                 calibrate_page_geometry: bool = True, calibration_samples: int = 3):
        self.target_capacity_keys = target_capacity_keys
        self.memory_budget_bytes = memory_budget_bytes
        self.entries_per_page = entries_per_page
        self.max_pages = max_pages
        self.workload = workload
        self.calibrate_page_geometry = calibrate_page_geometry
        self.calibration_samples = calibration_samples


class AutoStorage:
    """Accepted for API compatibility (sparse_embedding/__init__.py:63-78); the
    GPU store keeps every row in HBM and never spills."""

    def __init__(self, memory_limit_bytes=None, spill_directory=None, max_spill_bytes=None,
                 high_watermark=None, low_watermark=None):
        self.memory_limit_bytes = memory_limit_bytes
        self.spill_directory = None if spill_directory is None else os.fspath(spill_directory)


class MemoryOnly:
    """sparse_embedding/__init__.py:81-84."""


class EmbeddingConfig:
    """se::EmbeddingConfig (interface/embedding_config.hpp:31-43; __init__.py:105-135)
    plus the device the store lives on."""

    def __init__(
        self,
        dims: Sequence[int],
        thread_budget: int = 0,
        value_dtype: Any = "float32",
        optimizer_dtype: Any = "",
        gradient_dtype: Any = "",
        gradient_scale: float = 1.0,
        key_dtype: Any = "int64",
        storage: AutoStorage | MemoryOnly | None = None,
        storage_tuning: StorageTuningOptions | None = None,
        enable_optimizer: bool = True,
        device: int | None = None,
        initial_capacity: int = 0,
        simd_width: int = 16,
        accumulation: str = "ordered",
    ):
        self.dims = [int(d) for d in dims]
        self.thread_budget = int(thread_budget)
        self.value_dtype = _to_str(value_dtype)
        self.optimizer_dtype = _to_str(optimizer_dtype)
        self.gradient_dtype = _to_str(gradient_dtype)
        self.gradient_scale = float(gradient_scale)
        self.key_dtype = _to_str(key_dtype)
        self.storage = AutoStorage() if storage is None else storage
        self.storage_tuning = StorageTuningOptions() if storage_tuning is None else storage_tuning
        self.enable_optimizer = bool(enable_optimizer)
        self.device = device
        self.initial_capacity = int(initial_capacity)
        self.simd_width = int(simd_width)
        # How gradients are summed until optimizer_step (GPU store only):
        # "ordered" keeps every row and sums each key's rows in arrival order
        # (the reference's order); "atomic" adds them into per-key fp32 sums as
        # they arrive (vector reductions; the order of the adds varies).
        self.accumulation = str(accumulation)


class Initializer:
    kind = "zeros"
    min_val = 0.0
    max_val = 0.0


class Zeros(Initializer):
    """ZerosInitializer (initializer/zeros_initializer.hpp:27-31)."""

    kind = "zeros"


class Uniform(Initializer):
    """UniformInitializer (initializer/uniform_initializer.hpp:29-54): deterministic
    per key, bit-identical to simd_uniform_init."""

    kind = "uniform"

    def __init__(self, min_val: float = -0.05, max_val: float = 0.05):
        self.min_val = float(min_val)
        self.max_val = float(max_val)


class Optimizer:
    kind = "none"


# ---------------------------------------------------------------------------
# Dynamic learning-rate policies (optimizer/dynamic_lr_policy.hpp:32-124,
# bindings/module.cpp:491-560): the row's learning rate from its score
# ---------------------------------------------------------------------------


class LrPolicy:
    code = 0
    requires_score = False
    min_lr_ratio = 0.0
    max_score = 0
    lut: list = []


class ConstantLrPolicy(LrPolicy):
    """lr for every row."""


class SqrtDecayLrPolicy(LrPolicy):
    """lr / sqrt(score) (lr at score 0)."""

    code = 1
    requires_score = True


class LogDecayLrPolicy(LrPolicy):
    """lr / log2(2 + score)."""

    code = 2
    requires_score = True


class InverseDecayLrPolicy(LrPolicy):
    """lr / score (lr at score 0)."""

    code = 3
    requires_score = True


class CosineFrequencyLrPolicy(LrPolicy):
    """From lr at score 0 down to min_lr_ratio * lr at max_score along a half cosine."""

    code = 4
    requires_score = True

    def __init__(self, min_lr_ratio: float = 0.1, max_score: int = 1024):
        if not math.isfinite(min_lr_ratio) or min_lr_ratio < 0.0 or min_lr_ratio > 1.0:
            raise ValueError("min_lr_ratio must be finite and in [0, 1]")
        if int(max_score) == 0:
            raise ValueError("max_score must be greater than zero")
        self.min_lr_ratio = float(min_lr_ratio)
        self.max_score = int(max_score)


class CustomLutLrPolicy(LrPolicy):
    """lr * lut[min(score, len(lut) - 1)]."""

    code = 5
    requires_score = True

    def __init__(self, lut):
        lut = [float(x) for x in lut]
        if not lut:
            raise ValueError("lut must not be empty")
        if any(not math.isfinite(x) or x < 0.0 for x in lut):
            raise ValueError("lut multipliers must be finite and non-negative")
        self.lut = lut


def _check_policy(policy):
    if policy is not None and not isinstance(policy, LrPolicy):
        raise TypeError("dynamic_lr_policy must be an LrPolicy")
    return policy


class Sgd(Optimizer):
    """SgdConfig (optimizer/optimizer_config.hpp:38-42): p -= lr * (g + wd * p)."""

    kind = "sgd"

    def __init__(self, lr: float = 1e-2, weight_decay: float = 0.0, dynamic_lr_policy=None):
        self.dynamic_lr_policy = _check_policy(dynamic_lr_policy)
        self.lr = float(lr)
        self.weight_decay = float(weight_decay)


class Adam(Optimizer):
    """AdamConfig (optimizer_config.hpp:28-36) with per-row step counters
    (optimizer/adam_optimizer.hpp:138-165)."""

    kind = "adam"

    def __init__(self, lr: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                 weight_decay: float = 0.0, dynamic_lr_policy=None):
        self.dynamic_lr_policy = _check_policy(dynamic_lr_policy)
        self.lr = float(lr)
        self.beta1 = float(beta1)
        self.beta2 = float(beta2)
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)


class Adagrad(Optimizer):
    """Adagrad, an addition of the GPU store (the reference has none).

    The accumulator of a row starts at `initial_accumulator_value` when the row
    is created; each step: g += wd * p (when wd > 0), acc += g * g,
    p -= lr * g / (sqrt(acc) + eps), with the fused rounding the kernel and the
    oracle share.
    """

    kind = "adagrad"

    def __init__(self, lr: float = 1e-2, eps: float = 1e-8, weight_decay: float = 0.0,
                 initial_accumulator_value: float = 0.1, dynamic_lr_policy=None):
        self.dynamic_lr_policy = _check_policy(dynamic_lr_policy)
        self.lr = float(lr)
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)
        self.initial_accumulator_value = float(initial_accumulator_value)


# ---------------------------------------------------------------------------
# Store
# ---------------------------------------------------------------------------


def _default_device() -> int:
    from ._tensors import torch_mod

    torch = torch_mod()
    if not torch.cuda.is_available():
        raise RuntimeError("the GPU store needs a CUDA device")
    return torch.cuda.current_device()


def _float_list(arr) -> list:
    """Values of a host array (float32, float16, or bfloat16 as a torch tensor) as Python floats."""
    if arr is None:
        return []
    if hasattr(arr, "float") and hasattr(arr, "numpy"):  # torch bfloat16
        arr = arr.float().numpy()
    return np.asarray(arr, dtype=np.float32).reshape(-1).tolist()


def _from_float_list(values, shape, dtype_name: str):
    """Floats as an array of a store dtype (bfloat16 as a torch tensor)."""
    a = np.asarray(values, dtype=np.float32).reshape(shape)
    if dtype_name == "float16":
        return a.astype(np.float16)
    if dtype_name == "bfloat16":
        from ._tensors import torch_mod

        return torch_mod().from_numpy(a).to(torch_mod().bfloat16)
    return a


class EmbeddingStore:
    """GPU store with the reference EmbeddingStore's hot-path API
    (sparse_embedding/src/bindings/module.cpp:611-724)."""

    def __init__(self, embedding_config: EmbeddingConfig, initializer_config: Initializer | None = None,
                 optimizer_config: Optimizer | None = None, score_policy: str = "none"):
        cfg = embedding_config
        # EmbeddingStoreWrapper constructor checks (module.cpp:103-190)
        value_dtype = _parse_value_dtype(cfg.value_dtype, "dtype")
        optimizer_dtype = _parse_value_dtype(cfg.optimizer_dtype or cfg.value_dtype, "opt_dtype")
        gradient_dtype = _parse_value_dtype(cfg.gradient_dtype or cfg.value_dtype, "gradient_dtype")
        key_dtype = _parse_key_dtype(cfg.key_dtype)
        init = initializer_config if initializer_config is not None else Uniform(-0.05, 0.05)
        if not cfg.enable_optimizer and optimizer_config is not None:
            raise ValueError("optimizer_config cannot be provided when enable_optimizer is false")
        opt = optimizer_config
        if cfg.enable_optimizer and opt is None:
            opt = Adam()
        if not cfg.dims:
            raise ValueError("dims must not be empty")
        # parse_store_score_policy (backend/hogwild/store_construction.cpp:9-19)
        if score_policy not in ("none", "lfu", "lru", "manual"):
            raise ValueError(f"unknown score policy: {score_policy}")
        policy = getattr(opt, "dynamic_lr_policy", None) if cfg.enable_optimizer else None
        if policy is not None and policy.requires_score and score_policy == "none":
            raise ValueError("dynamic learning-rate policy requires a score policy")
        if not math.isfinite(cfg.gradient_scale) or cfg.gradient_scale <= 0.0:
            raise ValueError("gradient_scale must be finite and greater than zero")
        accumulation = getattr(cfg, "accumulation", "ordered")
        if accumulation not in N.ACCUM_CODES:
            raise ValueError("accumulation must be 'ordered' or 'atomic'")
        self._config = cfg
        self._key_dtype = key_dtype
        self._value_dtype = value_dtype
        self._optimizer_dtype = optimizer_dtype
        self._gradient_dtype = gradient_dtype
        self._optimizer_enabled = cfg.enable_optimizer
        self._score_policy = score_policy
        self._thread_budget = cfg.thread_budget if cfg.thread_budget > 0 else max(1, os.cpu_count() or 1)
        self._device = _default_device() if cfg.device is None else int(cfg.device)
        self._lens_cache = {}  # dim -> one-element int64 device tensor (row_lengths of device batches)
        self._operational = True

        dims = (C.c_int64 * len(cfg.dims))(*cfg.dims)
        c = N.StoreConfig()
        c.dims = C.cast(dims, C.POINTER(C.c_int64))
        c.num_dims = len(cfg.dims)
        c.key_dtype = N.KEY_CODES[key_dtype]
        c.value_dtype = N.VALUE_CODES[value_dtype]
        c.optimizer_dtype = N.VALUE_CODES[optimizer_dtype]
        c.gradient_dtype = N.VALUE_CODES[gradient_dtype]
        c.gradient_scale = cfg.gradient_scale
        c.enable_optimizer = int(cfg.enable_optimizer)
        c.init_kind = N.INIT_CODES[init.kind]
        c.init_min = init.min_val
        c.init_max = init.max_val
        kind = opt.kind if (cfg.enable_optimizer and opt is not None) else "none"
        c.optimizer_kind = N.OPT_CODES[kind]
        c.lr = getattr(opt, "lr", 0.0)
        c.beta1 = getattr(opt, "beta1", 0.9)
        c.beta2 = getattr(opt, "beta2", 0.999)
        c.eps = getattr(opt, "eps", 1e-8)
        c.weight_decay = getattr(opt, "weight_decay", 0.0)
        c.initial_accumulator = getattr(opt, "initial_accumulator_value", 0.0)
        cap = cfg.initial_capacity or int(getattr(cfg.storage_tuning, "target_capacity_keys", 0) or 0)
        c.initial_capacity = cap
        c.device = self._device
        c.simd_width = cfg.simd_width
        c.internal_shards = self._thread_budget
        c.score_policy = {"none": 0, "lfu": 1, "lru": 2, "manual": 3}[score_policy]
        c.accumulation = N.ACCUM_CODES[accumulation]
        lut = None
        if policy is not None:
            c.lr_policy = policy.code
            c.lr_min_ratio = policy.min_lr_ratio
            c.lr_max_score = policy.max_score
            if policy.lut:
                lut = (C.c_float * len(policy.lut))(*policy.lut)
                c.lr_lut = C.cast(lut, C.POINTER(C.c_float))
                c.lr_lut_len = len(policy.lut)
        self._optimizer = opt
        self._lib = N.lib()
        h = C.c_void_p()
        N.check(self._lib.se_store_create(C.byref(c), C.byref(h)))
        self._h = h

    def __del__(self):
        pool = getattr(self, "_async_pool", None)
        if pool is not None:
            pool.shutdown(wait=True)
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                self._lib.se_store_destroy(h)
            except Exception:
                pass
            self._h = None

    # ---- helpers -------------------------------------------------------------

    def _keys(self, keys) -> Arr:
        k = as_input(keys, "keys")
        if len(k.shape) > 1:
            raise ValueError("keys must be a 1D tensor")
        if k.dtype != self._key_dtype:
            # validate_key_dtype (bindings/module_wrapper.hpp:77-84)
            raise ValueError(
                f"key dtype does not match store key_dtype: expected {self._key_dtype}, got {k.dtype}")
        self._check_device(k)
        return k

    def _check_device(self, a: Arr) -> None:
        if a.cuda_device is not None and a.cuda_device != self._device:
            raise ValueError(f"tensor is on cuda:{a.cuda_device}, the store on cuda:{self._device}")

    @staticmethod
    def _stream(a: Arr):
        return C.c_void_p(a.stream) if a.stream else None

    def _check_operational(self):
        if not self._operational:
            raise RuntimeError("store is in terminal failure state")

    # ---- hot path ------------------------------------------------------------

    def _lookup(self, keys, dim: int, insert: bool):
        self._check_operational()
        dim = int(dim)
        if dim <= 0:
            raise ValueError("dim must be > 0")
        k = self._keys(keys)
        n = k.size
        out = empty_like_space(k, (n * dim,), self._value_dtype)
        lens = np.full(n, dim, dtype=np.int64) if k.cuda_device is None else None
        fn = self._lib.se_lookup_or_insert_dim if insert else self._lib.se_forward_lookup_dim
        N.check(fn(self._h, k.ptr, n, dim, data_ptr(out), self._stream(k)))
        if lens is None:
            lens = self._device_lens(n, dim)
        return out, lens

    def _device_lens(self, n: int, dim: int):
        """row_lengths of a device batch: every row has `dim` values. A
        broadcast view (stride 0) of one cached element per dim, so the call
        launches no fill kernel between the library's kernels; torch rejects
        in-place writes to such a view, so the shared element cannot be
        changed through it."""
        from ._tensors import torch_mod

        torch = torch_mod()
        one = self._lens_cache.get(dim)
        if one is None:
            one = torch.full((1,), dim, dtype=torch.int64, device=f"cuda:{self._device}")
            self._lens_cache[dim] = one
        return one.expand(n)

    def lookup(self, keys, dim: int):
        """forward_lookup: (values[n*dim], row_lengths[n]); absent keys read as zeros."""
        return self._lookup(keys, dim, insert=False)

    def forward_lookup(self, keys, dim: int):
        return self._lookup(keys, dim, insert=False)

    def lookup_or_insert(self, keys, dim: int):
        """Inserts absent keys (initialised from the key), then returns their rows."""
        return self._lookup(keys, dim, insert=True)

    def accumulate_gradients(self, keys, grads) -> None:
        # EmbeddingStoreWrapper::accumulate_gradients (module_wrapper_methods.inl:165-172)
        if not self._optimizer_enabled:
            raise RuntimeError("accumulate_gradients requires optimizer enabled")
        self._check_operational()
        k = self._keys(keys)
        g = as_input(grads, "grads")
        self._check_device(g)
        n = k.size
        # SyncOpsImpl::accumulate_gradients shape rules (module_typed_sync.inl:129-166)
        if len(g.shape) == 2:
            if g.shape[0] != n:
                raise ValueError("grads shape[0] must match keys length")
            dim = int(g.shape[1])
        elif len(g.shape) == 1:
            dim = 0
            if n > 0:
                if g.shape[0] % n != 0:
                    raise ValueError("1D grads length must be a multiple of keys length")
                dim = int(g.shape[0]) // n
        else:
            raise ValueError("grads must be a 1D or 2D tensor")
        if g.dtype != self._gradient_dtype:
            raise ValueError("dtype mismatch in dlpack_to_span")
        if (k.cuda_device is None) != (g.cuda_device is None):
            raise ValueError("keys and grads must be in the same memory space")
        if n == 0:
            return
        stream = self._stream(g) or self._stream(k)
        N.check(self._lib.se_accumulate_gradients_dim(self._h, k.ptr, n, dim, g.ptr, stream))

    # ---- embedding bag ------------------------------------------------------------

    def _offsets(self, offsets, k: Arr, what: str = "offsets") -> Arr:
        o = as_input(offsets, what)
        if len(o.shape) != 1 or o.size < 1:
            raise ValueError("offsets must be a 1D tensor of num_bags + 1 entries")
        if o.dtype != "int64":
            raise ValueError("offsets must be int64")
        if (o.cuda_device is None) != (k.cuda_device is None):
            raise ValueError("keys and offsets must be in the same memory space")
        return o

    def embedding_bag(self, keys, offsets, dim: int, insert: bool = True):
        """Sum-pooled rows of multi-hot bags: out[b] = sum of the rows of
        keys[offsets[b]:offsets[b+1]] in key order (fp32 adds, rounded once to
        the value dtype). With insert, absent keys are inserted first
        (lookup_or_insert); else they add zero rows. Returns [num_bags, dim]."""
        self._check_operational()
        dim = int(dim)
        if dim <= 0:
            raise ValueError("dim must be > 0")
        k = self._keys(keys)
        o = self._offsets(offsets, k)
        nb = o.size - 1
        out = empty_like_space(k, (nb, dim), self._value_dtype)
        N.check(self._lib.se_embedding_bag(self._h, k.ptr, k.size, o.ptr, nb, dim, data_ptr(out), int(bool(insert)),
                                           self._stream(k)))
        return out

    def embedding_bag_backward(self, keys, offsets, pooled_grads) -> None:
        """Accumulates pooled_grads[b] (gradient dtype, [num_bags, dim]) as the
        gradient of every key of bag b."""
        if not self._optimizer_enabled:
            raise RuntimeError("accumulate_gradients requires optimizer enabled")
        self._check_operational()
        k = self._keys(keys)
        o = self._offsets(offsets, k)
        g = as_input(pooled_grads, "grads")
        self._check_device(g)
        nb = o.size - 1
        if len(g.shape) != 2 or g.shape[0] != nb:
            raise ValueError("pooled_grads must be [num_bags, dim]")
        if g.dtype != self._gradient_dtype:
            raise ValueError("dtype mismatch in dlpack_to_span")
        if (k.cuda_device is None) != (g.cuda_device is None):
            raise ValueError("keys and grads must be in the same memory space")
        stream = self._stream(g) or self._stream(k)
        N.check(self._lib.se_embedding_bag_backward(self._h, k.ptr, k.size, o.ptr, nb, int(g.shape[1]), g.ptr,
                                                    stream))

    # ---- scores ---------------------------------------------------------------------

    def assign_scores(self, keys, scores) -> None:
        """Sets each key's score in the first table holding it; absent keys are
        skipped (hogwild_embedding_store.hpp:5202-5250)."""
        k = self._keys(keys)
        sc = as_input(scores, "scores")
        if sc.dtype != "uint64":
            raise ValueError("scores must be uint64")
        if sc.size != k.size:
            raise ValueError("assign_scores row counts differ")
        if (k.cuda_device is None) != (sc.cuda_device is None):
            raise ValueError("keys and scores must be in the same memory space")
        N.check(self._lib.se_assign_scores(self._h, k.ptr, k.size, sc.ptr, self._stream(k)))

    def read_scores(self, keys):
        """uint64 score of each key (0 when absent); host keys give a numpy array."""
        k = self._keys(keys)
        out = empty_like_space(k, (k.size,), "uint64")
        if k.size:
            N.check(self._lib.se_read_scores(self._h, k.ptr, k.size, data_ptr(out), self._stream(k)))
        return out

    # ---- mutation API -----------------------------------------------------------

    def assign(self, keys, values) -> None:
        """Sets the parameters of each key (inserting absent keys with fresh
        optimizer state); keys must be distinct. SyncOpsImpl::assign shape rules
        (bindings/typed/module_typed_sync.inl:92-126)."""
        self._check_operational()
        k = self._keys(keys)
        v = as_input(values, "values")
        self._check_device(v)
        n = k.size
        if len(v.shape) == 2:
            if v.shape[0] != n:
                raise ValueError("values shape[0] must match keys length")
            dim = int(v.shape[1])
        elif len(v.shape) == 1:
            dim = 0
            if n > 0:
                if v.shape[0] % n != 0:
                    raise ValueError("1D values length must be a multiple of keys length")
                dim = int(v.shape[0]) // n
        else:
            raise ValueError("values must be a 1D or 2D tensor")
        if v.dtype != self._value_dtype:
            raise ValueError("dtype mismatch in dlpack_to_span")
        if (k.cuda_device is None) != (v.cuda_device is None):
            raise ValueError("keys and values must be in the same memory space")
        if n == 0:
            return
        stream = self._stream(v) or self._stream(k)
        N.check(self._lib.se_assign_dim(self._h, k.ptr, n, dim, v.ptr, stream))

    def contains(self, keys):
        """uint8 per key: 1 when any table holds it (module_wrapper_methods.inl:143-160)."""
        k = self._keys(keys)
        n = k.size
        out = empty_like_space(k, (n,), "uint8")
        if n:
            N.check(self._lib.se_contains(self._h, k.ptr, n, data_ptr(out), self._stream(k)))
        return out

    def erase(self, keys) -> None:
        """Removes the keys from every table; absent keys are ignored."""
        k = self._keys(keys)
        N.check(self._lib.se_erase(self._h, k.ptr, k.size, self._stream(k)))

    def erase_dimension(self, keys, dimension: int) -> None:
        """Removes the keys from the table of one dim (module_wrapper_methods.inl:195-210)."""
        if int(dimension) < 0:
            raise ValueError("erase dimension must be non-negative")
        k = self._keys(keys)
        N.check(self._lib.se_erase_dimension(self._h, int(dimension), k.ptr, k.size, self._stream(k)))

    def optimizer_step(self, normalization_steps: int, stream: int | None = None) -> None:
        # EmbeddingStoreWrapper::optimizer_step (module_wrapper_methods.inl:174-180)
        if not self._optimizer_enabled:
            raise RuntimeError("optimizer_step requires optimizer enabled")
        self._check_operational()
        if isinstance(normalization_steps, bool) or int(normalization_steps) < 0:
            raise TypeError("normalization_steps must be a non-negative integer")
        if stream is None:
            stream = self._current_stream()
        N.check(self._lib.se_optimizer_step(self._h, int(normalization_steps),
                                            C.c_void_p(stream) if stream else None))

    def clear(self) -> None:
        """Removes every key and discards the gradients accumulated since the
        last optimizer_step (EmbeddingStoreWrapper::clear,
        module_wrapper_methods.inl:212-216); reserved capacity is kept."""
        self._check_operational()
        stream = self._current_stream()
        N.check(self._lib.se_store_clear(self._h, C.c_void_p(stream) if stream else None))

    # ---- asyncio variants (module.cpp:648-684) --------------------------------
    # Each returns an asyncio future of the running loop (the reference's
    # create_asyncio_future, bindings/async_bridge.hpp:74-87). The call runs on
    # the store's worker thread on the caller's CUDA stream; the future
    # completes with the synchronous method's result once the device work of
    # the call has finished, or with its exception. Argument checks that the
    # reference makes before dispatching raise immediately.

    def _async(self, fn, *args):
        import asyncio
        from concurrent.futures import ThreadPoolExecutor

        loop = asyncio.get_running_loop()
        if getattr(self, "_async_pool", None) is None:
            self._async_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="se-async")
        from ._tensors import _TORCH

        stream = None
        if _TORCH is not None and _TORCH.cuda.is_available() and _TORCH.cuda.is_initialized():
            stream = _TORCH.cuda.current_stream(self._device)

        def work():
            if stream is None:
                out = fn(*args)
            else:
                with _TORCH.cuda.stream(stream):
                    out = fn(*args)
            self.synchronize()  # the call's device work is done; deferred errors raise here
            return out

        return loop.run_in_executor(self._async_pool, work)

    def async_lookup(self, keys, dim: int):
        if int(dim) <= 0:
            raise ValueError("dim must be > 0")
        return self._async(self.lookup, keys, dim)

    def async_lookup_or_insert(self, keys, dim: int):
        if int(dim) <= 0:
            raise ValueError("dim must be > 0")
        return self._async(self.lookup_or_insert, keys, dim)

    def async_assign(self, keys, values):
        return self._async(self.assign, keys, values)

    def async_accumulate_gradients(self, keys, grads):
        if not self._optimizer_enabled:
            raise RuntimeError("async_accumulate_gradients requires optimizer enabled")
        return self._async(self.accumulate_gradients, keys, grads)

    def async_optimizer_step(self, normalization_steps: int):
        if not self._optimizer_enabled:
            raise RuntimeError("async_optimizer_step requires optimizer enabled")
        return self._async(self.optimizer_step, normalization_steps)

    def async_contains(self, keys):
        return self._async(self.contains, keys)

    def async_erase(self, keys):
        return self._async(self.erase, keys)

    def async_clear(self):
        return self._async(self.clear)

    def async_assign_scores(self, keys, scores):
        return self._async(self.assign_scores, keys, scores)

    def _current_stream(self) -> int | None:
        from ._tensors import _TORCH

        if _TORCH is not None and _TORCH.cuda.is_available() and _TORCH.cuda.is_initialized():
            return _TORCH.cuda.current_stream(self._device).cuda_stream
        return None

    # ---- metadata ------------------------------------------------------------

    def total_size(self) -> int:
        out = C.c_uint64()
        N.check(self._lib.se_store_size(self._h, C.byref(out)))
        return int(out.value)

    def size(self, dim: int | None = None) -> int:
        if dim is None:
            return self.total_size()
        out = C.c_uint64()
        N.check(self._lib.se_store_dim_size(self._h, int(dim), C.byref(out)))
        return int(out.value)

    def max_dim(self) -> int:
        return max(self._config.dims)

    def num_slots(self) -> int:
        return len(set(self._config.dims))

    def table_dims(self) -> list[int]:
        return sorted(set(self._config.dims))

    def internal_shard_count(self) -> int:
        out = C.c_uint64()
        N.check(self._lib.se_store_internal_shard_count(self._h, C.byref(out)))
        return int(out.value)

    @property
    def entries_per_page(self) -> int:
        out = C.c_uint64()
        N.check(self._lib.se_store_entries_per_page(self._h, C.byref(out)))
        return int(out.value)

    def reserve(self, keys_count: int, dim: int) -> None:
        if int(dim) <= 0:
            raise ValueError("dim must be > 0")
        N.check(self._lib.se_store_reserve(self._h, int(keys_count), int(dim)))

    def reserve_per_shard(self, counts: Sequence[int], dim: int) -> None:
        if int(dim) <= 0:
            raise ValueError("dim must be > 0")
        if len(counts) != self.internal_shard_count():
            raise ValueError("counts size mismatch")
        self.reserve(int(sum(counts)), dim)

    def key_dtype(self) -> str:
        return self._key_dtype

    def value_dtype(self) -> str:
        return self._value_dtype

    def optimizer_dtype(self) -> str:
        return self._optimizer_dtype

    def gradient_dtype(self) -> str:
        return self._gradient_dtype

    def optimizer_enabled(self) -> bool:
        return self._optimizer_enabled

    def score_policy(self) -> str:
        return self._score_policy

    def device(self) -> int:
        return self._device

    def dropped_gradients(self) -> int:
        out = C.c_uint64()
        N.check(self._lib.se_store_dropped_gradients(self._h, C.byref(out)))
        return int(out.value)

    def synchronize(self) -> None:
        N.check(self._lib.se_store_synchronize(self._h))

    def storage_stats(self) -> dict:
        return {"backend": "b200-hbm", "device": self._device, "total_size": self.total_size(),
                "dropped_gradients": self.dropped_gradients()}

    def device_stats(self) -> dict:
        return self.storage_stats()

    def mark_terminal_failure(self) -> None:
        self._operational = False

    def is_operational(self) -> bool:
        return self._operational

    def read_state(self, key: int, dim: int):
        """(found, param, state, step) of one key, for checks. Arrays hold raw
        values of the value / optimizer dtypes (uint16 bits for 16-bit types)."""
        nstate = {"adam": 2, "adagrad": 1}.get(getattr(self._optimizer, "kind", "none"), 0)
        if not self._optimizer_enabled:
            nstate = 0
        vt = np.float32 if self._value_dtype == "float32" else np.uint16
        ot = np.float32 if self._optimizer_dtype == "float32" else np.uint16
        p = np.zeros(dim, dtype=vt)
        s = np.zeros(max(1, nstate * dim), dtype=ot)
        step = C.c_uint32()
        found = C.c_int32()
        ukey = int(key) & 0xFFFFFFFFFFFFFFFF
        N.check(self._lib.se_store_read_state(self._h, int(dim), ukey, p.ctypes.data, s.ctypes.data,
                                              C.byref(step), C.byref(found)))
        return bool(found.value), p, s[: nstate * dim], int(step.value)

    def profile(self, enable: bool = True) -> None:
        N.check(self._lib.se_store_profile_enable(self._h, int(enable)))

    def profile_read(self, name: str) -> tuple[float, int]:
        ms = C.c_double()
        cnt = C.c_uint64()
        N.check(self._lib.se_store_profile_read(self._h, name.encode(), C.byref(ms), C.byref(cnt)))
        return float(ms.value), int(cnt.value)

    # ---- conventions the GPU store does not provide --------------------------

    def export_page_images(self):
        """Page images of every table (EmbeddingStoreWrapper::export_page_images,
        module_wrapper_methods.inl:254-290): a list of dicts with the
        reference's fields. The GPU store has no host pages; page p of a
        table holds entries [p * E, (p + 1) * E) of its export in directory
        order, E = entries_per_page; slot_ordinals are the entries' places
        in the page and page_slot_stride_bytes is the reference's slot stride
        for the row (row bytes rounded up to 64). values / optimizer_states
        are float lists (row-major), steps the Adam steps (0 otherwise),
        scores the keys' scores (0 without a score policy), seq_counts 0."""
        from .checkpoint import export_batches

        per_page = self.entries_per_page
        vb = 4 if self._value_dtype == "float32" else 2
        pages = []
        for dim, keys, values, states, steps in export_batches(self, batch_size=per_page,
                                                               include_optimizer_state=True, include_steps=True):
            scores = self.read_scores(keys) if self._score_policy != "none" else np.zeros(len(keys), np.uint64)
            pages.append({
                "embedding_dim": int(dim),
                "physical_page_id": sum(1 for q in pages if q["embedding_dim"] == int(dim)),
                "page_slot_stride_bytes": (int(dim) * vb + 63) // 64 * 64,
                "slot_ordinals": list(range(len(keys))),
                "keys": [int(k) & 0xFFFFFFFFFFFFFFFF for k in np.asarray(keys).tolist()],
                "seq_counts": [0] * len(keys),
                "scores": [int(x) for x in np.asarray(scores).tolist()],
                "steps": [int(x) for x in np.asarray(steps).tolist()],
                "values": _float_list(values),
                "optimizer_states": _float_list(states),
            })
        return pages

    def import_page_images(self, pages):
        """Loads page images into this (empty) store (import_page_images,
        hogwild_embedding_store.hpp:6512-6590): every page's keys get their
        values, optimizer state, Adam steps and scores. Errors as the
        reference: a dimension without a table, repeated page ids of a
        dimension, or a store that already holds keys."""
        from .checkpoint import assign_opt_state

        self._check_operational()
        dims = set(self._config.dims)
        seen = set()
        for page in pages:
            d = int(page["embedding_dim"])
            if d not in dims:
                raise ValueError("page-image import dimension has no physical table")
            if (d, int(page["physical_page_id"])) in seen:
                raise ValueError("page-image import has duplicate page ids")
            seen.add((d, int(page["physical_page_id"])))
        if self.total_size() != 0:
            raise RuntimeError("page-image import requires empty slots")
        kdt = np.dtype(self._key_dtype)
        ns = {"adam": 2, "adagrad": 1}.get(getattr(self._optimizer, "kind", "none"), 0) \
            if self._optimizer_enabled else 0
        for page in pages:
            d = int(page["embedding_dim"])
            n = len(page["keys"])
            if n == 0:
                continue
            keys = np.asarray(page["keys"], dtype=np.uint64).view(np.int64).astype(kdt) if kdt.kind == "i" \
                else np.asarray(page["keys"], dtype=np.uint64).astype(kdt)
            values = _from_float_list(page["values"], (n, d), self._value_dtype)
            self.assign(keys, values)
            if ns:
                states = _from_float_list(page["optimizer_states"], (n, ns * d), self._optimizer_dtype)
                assign_opt_state(self, keys, states, d, steps=np.asarray(page["steps"], dtype=np.uint32))
            if self._score_policy != "none" and any(page["scores"]):
                self.assign_scores(keys, np.asarray(page["scores"], dtype=np.uint64))
