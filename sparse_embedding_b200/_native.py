"""ctypes binding of libse_gpu.so (the C ABI declared in include/se_gpu.h).

The library is the only compute path of this package: if it is missing or
fails to load, every operation raises instead of falling back to anything
else.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from .build import LIB_PATH

SE_OK = 0
SE_ERR_INVALID_ARGUMENT = -1
SE_ERR_RUNTIME = -2
SE_ERR_OVERFLOW = -3
SE_ERR_CUDA = -4
SE_ERR_OUT_OF_MEMORY = -5
SE_ERR_TABLE_FULL = -6
SE_ERR_NOT_IMPLEMENTED = -7

KEY_CODES = {"int32": 0, "uint32": 1, "int64": 2, "uint64": 3}
VALUE_CODES = {"float32": 0, "float16": 1, "bfloat16": 2}
OPT_CODES = {"none": 0, "sgd": 1, "adam": 2, "adagrad": 3}
INIT_CODES = {"zeros": 0, "uniform": 1}
PART_CODES = {"modulo": 0, "hash": 1, "fast_range": 2}
ACCUM_CODES = {"ordered": 0, "atomic": 1}


class StoreConfig(C.Structure):
    """Mirror of se_store_config."""

    _fields_ = [
        ("dims", C.POINTER(C.c_int64)),
        ("num_dims", C.c_size_t),
        ("key_dtype", C.c_int32),
        ("value_dtype", C.c_int32),
        ("optimizer_dtype", C.c_int32),
        ("gradient_dtype", C.c_int32),
        ("gradient_scale", C.c_float),
        ("enable_optimizer", C.c_int32),
        ("init_kind", C.c_int32),
        ("init_min", C.c_float),
        ("init_max", C.c_float),
        ("optimizer_kind", C.c_int32),
        ("lr", C.c_float),
        ("beta1", C.c_float),
        ("beta2", C.c_float),
        ("eps", C.c_float),
        ("weight_decay", C.c_float),
        ("initial_accumulator", C.c_float),
        ("initial_capacity", C.c_uint64),
        ("device", C.c_int32),
        ("simd_width", C.c_int32),
        ("internal_shards", C.c_int32),
        ("score_policy", C.c_int32),
        ("lr_policy", C.c_int32),
        ("lr_min_ratio", C.c_float),
        ("lr_max_score", C.c_uint64),
        ("lr_lut", C.POINTER(C.c_float)),
        ("lr_lut_len", C.c_size_t),
        ("accumulation", C.c_int32),
    ]


_vp = C.c_void_p
_sz = C.c_size_t
_i32 = C.c_int32
_i64 = C.c_int64
_u32 = C.c_uint32
_u64 = C.c_uint64

# name -> argtypes; every function returns int (status) unless listed in _RESTYPES.
_SIGNATURES = {
    "se_last_error": [],
    "se_version": [],
    "se_kernel_launch_count": [],
    "se_store_create": [C.POINTER(StoreConfig), C.POINTER(_vp)],
    "se_store_destroy": [_vp],
    "se_forward_lookup": [_vp, _vp, _sz, _vp, _sz, C.POINTER(_i64), _sz, _vp],
    "se_lookup_or_insert": [_vp, _vp, _sz, _vp, _sz, C.POINTER(_i64), _sz, _vp],
    "se_forward_lookup_dim": [_vp, _vp, _sz, _i64, _vp, _vp],
    "se_lookup_or_insert_dim": [_vp, _vp, _sz, _i64, _vp, _vp],
    "se_accumulate_gradients": [_vp, _vp, _sz, _vp, _sz, C.POINTER(_i64), _sz, _vp],
    "se_accumulate_gradients_dim": [_vp, _vp, _sz, _i64, _vp, _vp],
    "se_optimizer_step": [_vp, _sz, _vp],
    "se_contains": [_vp, _vp, _sz, _vp, _vp],
    "se_assign": [_vp, _vp, _sz, _vp, _sz, C.POINTER(_i64), _sz, _vp],
    "se_assign_dim": [_vp, _vp, _sz, _i64, _vp, _vp],
    "se_erase": [_vp, _vp, _sz, _vp],
    "se_embedding_bag": [_vp, _vp, _sz, _vp, _sz, _i64, _vp, _i32, _vp],
    "se_assign_scores": [_vp, _vp, _sz, _vp, _vp],
    "se_read_scores": [_vp, _vp, _sz, _vp, _vp],
    "se_export_snapshot": [_vp, _i64, C.POINTER(_u64), _vp],
    "se_export_read": [_vp, _i64, _u64, _u64, _vp, _vp, _vp, _vp, _vp],
    "se_assign_opt_states": [_vp, _i64, _vp, _sz, _vp, _sz, _vp, _vp],
    "se_embedding_bag_backward": [_vp, _vp, _sz, _vp, _sz, _i64, _vp, _vp],
    "se_erase_dimension": [_vp, _i64, _vp, _sz, _vp],
    "se_store_size": [_vp, C.POINTER(_u64)],
    "se_store_dim_size": [_vp, _i64, C.POINTER(_u64)],
    "se_store_reserve": [_vp, _sz, _i64],
    "se_store_internal_shard_count": [_vp, C.POINTER(_u64)],
    "se_store_entries_per_page": [_vp, C.POINTER(_u64)],
    "se_store_dropped_gradients": [_vp, C.POINTER(_u64)],
    "se_store_read_state": [_vp, _i64, _u64, _vp, _vp, C.POINTER(_u32), C.POINTER(_i32)],
    "se_store_synchronize": [_vp],
    "se_store_clear": [_vp, _vp],
    "se_store_profile_enable": [_vp, _i32],
    "se_store_profile_read": [_vp, C.c_char_p, C.POINTER(C.c_double), C.POINTER(_u64)],
    "se_partition": [_i32, _u32, _i32, _vp, _sz, _vp, _i32, _vp],
    "se_unique": [_i32, _vp, _sz, _vp, _vp, _vp, _vp, C.POINTER(_u64), _i32, _vp],
    "se_filter": [_i32, _u32, _i32, _vp, _sz, _u32, _vp, _i32, _vp],
    "se_partition_route": [_i32, _u32, _i32, _vp, _sz, _vp, _vp, _vp, _i32, _vp],
    "se_partition_route_noalloc": [_i32, _u32, _i32, _vp, _sz, _vp, _vp, _vp, _i32, _vp],
    "se_permute_rows": [_vp, _vp, _vp, _sz, _sz, _i32, _i32, _vp],
    "se_exchange_create": [_vp, _i32, _u32, _u32, _u64, _i64, _u32, C.POINTER(_vp)],
    "se_exchange_handle": [_vp, _vp, _sz],
    "se_exchange_connect": [_vp, _vp, _sz],
    "se_exchange_connect_local": [C.POINTER(_vp), _u32],
    "se_exchange_lookup": [_vp, _vp, _sz, _vp, _i32, _vp],
    "se_exchange_accumulate": [_vp, _vp, _sz, _vp, _vp],
    "se_exchange_accumulate_routed": [_vp, _vp, _sz, _vp],
    "se_exchange_check": [_vp, _vp],
    "se_exchange_set_dedupe": [_vp, _i32],
    "se_exchange_destroy": [_vp],
}
_RESTYPES = {"se_last_error": C.c_char_p, "se_version": C.c_char_p, "se_kernel_launch_count": _u64}

_lib = None
_lock = threading.Lock()


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def lib(path: Path | None = None):
    """Loads libse_gpu.so (once). Raises if it is absent: there is no fallback."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"libse_gpu.so not found at {p}; build it with "
                "`python -m sparse_embedding_b200.build` (nvcc, sm_100a)"
            )
        L = C.CDLL(str(p))
        for name, args in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, C.c_int)
        _lib = L
        return L


def check(rc: int) -> None:
    """Raises the Python exception that matches a C ABI status code."""
    if rc == SE_OK:
        return
    msg = (lib().se_last_error() or b"").decode()
    if rc == SE_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == SE_ERR_OVERFLOW:
        raise OverflowError(msg)
    if rc == SE_ERR_OUT_OF_MEMORY:
        raise MemoryError(msg)
    if rc == SE_ERR_NOT_IMPLEMENTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)
