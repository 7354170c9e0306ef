"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/libse_oracle.so`` (the scalar restatement in ``se_oracle.cpp``)
and, when it was built here, ``oracle/_ref/libse_ref.so`` (the reference's own
hot-path headers compiled in place by ``make -C oracle ref``). Only the tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module, and only as the checker or the timed CPU baseline.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
_LIB_PATH = ORACLE_DIR / "libse_oracle.so"
_REF_PATH = ORACLE_DIR / "_ref" / "libse_ref.so"

KEY_CODES = {"int32": 0, "uint32": 1, "int64": 2, "uint64": 3}
VALUE_CODES = {"float32": 0, "float16": 1, "bfloat16": 2}
OPT_CODES = {"none": 0, "sgd": 1, "adam": 2, "adagrad": 3}
INIT_CODES = {"zeros": 0, "uniform": 1}
PART_CODES = {"modulo": 0, "hash": 1, "fast_range": 2}

_c = ctypes
_vp = _c.c_void_p


def build(ref: bool = False) -> None:
    """Compile the oracle (and optionally the reference shim) with make."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "ref"], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = _c.CDLL(str(_LIB_PATH))
        L.or_last_error.restype = _c.c_char_p
        L.or_splitmix64.restype = _c.c_uint64
        L.or_splitmix64.argtypes = [_c.c_uint64]
        L.or_fmix32.restype = _c.c_uint32
        L.or_fmix32.argtypes = [_c.c_uint32]
        L.or_partition.argtypes = [_c.c_int, _c.c_uint32, _c.c_int, _vp, _c.c_size_t, _vp]
        L.or_filter.argtypes = [_c.c_int, _c.c_uint32, _c.c_int, _vp, _c.c_size_t, _c.c_uint32, _vp]
        L.or_uniform_init_f32.argtypes = [_vp, _c.c_size_t, _c.c_float, _c.c_float, _c.c_uint64, _c.c_int]
        L.or_sgd_f32.argtypes = [_vp, _vp, _c.c_float, _c.c_float, _c.c_size_t, _c.c_int]
        L.or_adam_f32.argtypes = [_vp, _vp, _vp, _vp] + [_c.c_float] * 7 + [_c.c_size_t, _c.c_int]
        L.or_adagrad_f32.argtypes = [_vp, _vp, _vp, _c.c_float, _c.c_float, _c.c_float, _c.c_size_t]
        L.or_f32_to_bf16.restype = _c.c_uint16
        L.or_f32_to_bf16.argtypes = [_c.c_float]
        L.or_f32_to_f16.restype = _c.c_uint16
        L.or_f32_to_f16.argtypes = [_c.c_float]
        L.or_store_create.restype = _vp
        L.or_store_create.argtypes = (
            [_vp, _c.c_size_t] + [_c.c_int] * 4 + [_c.c_float, _c.c_int, _c.c_int, _c.c_float, _c.c_float, _c.c_int]
            + [_c.c_float] * 6 + [_c.c_int, _c.c_int]
            + [_c.c_int, _c.c_int, _c.c_float, _c.c_uint64, _vp, _c.c_size_t]
        )
        L.or_store_destroy.argtypes = [_vp]
        L.or_store_reserve.argtypes = [_vp, _c.c_int64, _c.c_size_t]
        L.or_lookup.argtypes = [_vp, _vp, _c.c_size_t, _c.c_int64, _vp]
        L.or_lookup_or_insert.argtypes = [_vp, _vp, _c.c_size_t, _c.c_int64, _vp]
        L.or_accumulate_gradients.argtypes = [_vp, _vp, _c.c_size_t, _c.c_int64, _vp]
        L.or_optimizer_step.argtypes = [_vp, _c.c_size_t]
        L.or_store_size.restype = _c.c_uint64
        L.or_store_size.argtypes = [_vp, _c.c_int64]
        L.or_store_dropped.restype = _c.c_uint64
        L.or_store_dropped.argtypes = [_vp]
        L.or_read_row.argtypes = [_vp, _c.c_int64, _c.c_uint64, _vp, _vp, _vp]
        L.or_contains.argtypes = [_vp, _vp, _c.c_size_t, _vp]
        L.or_assign.argtypes = [_vp, _vp, _c.c_size_t, _c.c_int64, _vp]
        L.or_erase.argtypes = [_vp, _vp, _c.c_size_t, _c.c_int64]
        L.or_assign_scores.argtypes = [_vp, _vp, _c.c_size_t, _vp]
        L.or_read_scores.argtypes = [_vp, _vp, _c.c_size_t, _vp]
        _lib = L
    return _lib


def ref_available() -> bool:
    return _REF_PATH.exists()


def ref():
    """The reference's own compiled hot-path headers (oracle/_ref)."""
    global _ref
    if _ref is None:
        if not _REF_PATH.exists():
            raise FileNotFoundError(f"{_REF_PATH} not built (make -C oracle ref)")
        R = _c.CDLL(str(_REF_PATH))
        R.ref_partition.argtypes = [_c.c_int, _c.c_uint32, _c.c_int, _vp, _c.c_size_t, _vp]
        R.ref_filter.argtypes = [_c.c_int, _c.c_uint32, _c.c_int, _vp, _c.c_size_t, _c.c_uint32, _vp]
        R.ref_uniform_init_f32.argtypes = [_vp, _c.c_size_t, _c.c_float, _c.c_float, _c.c_uint64]
        R.ref_uniform_init_bf16.argtypes = [_vp, _c.c_size_t, _c.c_float, _c.c_float, _c.c_uint64]
        R.ref_uniform_init_f16.argtypes = [_vp, _c.c_size_t, _c.c_float, _c.c_float, _c.c_uint64]
        R.ref_sgd_f32.argtypes = [_vp, _vp, _c.c_float, _c.c_float, _c.c_size_t]
        R.ref_adam_f32.argtypes = [_vp, _vp, _vp, _vp] + [_c.c_float] * 7 + [_c.c_size_t]
        R.ref_accumulate_f32.argtypes = [_vp, _vp, _c.c_size_t]
        _ref = R
    return _ref


def _ptr(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def _check(rc: int) -> None:
    if rc != 0:
        msg = lib().or_last_error().decode()
        if rc == -3:
            raise OverflowError(msg)
        if rc == -2:
            raise RuntimeError(msg)
        raise ValueError(msg)


# ---------------------------------------------------------------------------
# Partitioners
# ---------------------------------------------------------------------------


def partition(kind: str, n: int, keys: np.ndarray) -> np.ndarray:
    keys = np.ascontiguousarray(keys)
    out = np.empty(len(keys), dtype=np.uint32)
    _check(lib().or_partition(PART_CODES[kind], n, KEY_CODES[keys.dtype.name], _ptr(keys), len(keys), _ptr(out)))
    return out


def filter_mask(kind: str, n: int, keys: np.ndarray, target: int) -> np.ndarray:
    keys = np.ascontiguousarray(keys)
    out = np.empty(len(keys), dtype=np.uint8)
    _check(lib().or_filter(PART_CODES[kind], n, KEY_CODES[keys.dtype.name], _ptr(keys), len(keys), target, _ptr(out)))
    return out.astype(bool)


def ref_partition(kind: str, n: int, keys: np.ndarray) -> np.ndarray:
    keys = np.ascontiguousarray(keys)
    out = np.empty(len(keys), dtype=np.uint32)
    rc = ref().ref_partition(PART_CODES[kind], n, KEY_CODES[keys.dtype.name], _ptr(keys), len(keys), _ptr(out))
    assert rc == 0
    return out


def ref_filter(kind: str, n: int, keys: np.ndarray, target: int) -> np.ndarray:
    keys = np.ascontiguousarray(keys)
    out = np.empty(len(keys), dtype=np.uint8)
    rc = ref().ref_filter(PART_CODES[kind], n, KEY_CODES[keys.dtype.name], _ptr(keys), len(keys), target, _ptr(out))
    assert rc == 0
    return out.astype(bool)


# ---------------------------------------------------------------------------
# Row arithmetic
# ---------------------------------------------------------------------------


def uniform_init(dim: int, key: int, lo: float = -0.05, hi: float = 0.05, simd_width: int = 16) -> np.ndarray:
    out = np.empty(dim, dtype=np.float32)
    lib().or_uniform_init_f32(_ptr(out), dim, lo, hi, key, simd_width)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    f = lib().or_f32_to_bf16
    return np.array([f(float(v)) for v in np.asarray(x, dtype=np.float32).ravel()], dtype=np.uint16)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    f = lib().or_f32_to_f16
    return np.array([f(float(v)) for v in np.asarray(x, dtype=np.float32).ravel()], dtype=np.uint16)


# ---------------------------------------------------------------------------
# Store flow
# ---------------------------------------------------------------------------


class OracleStore:
    """CPU restatement of the reference store's hot path (one table per dim)."""

    def __init__(
        self,
        dims,
        key_dtype="int64",
        value_dtype="float32",
        optimizer_dtype="",
        gradient_dtype="",
        gradient_scale=1.0,
        enable_optimizer=True,
        init="uniform",
        init_min=-0.05,
        init_max=0.05,
        optimizer="adam",
        lr=1e-3,
        beta1=0.9,
        beta2=0.999,
        eps=1e-8,
        weight_decay=0.0,
        initial_accumulator=0.0,
        simd_width=16,
        threads=1,
        score_policy="none",
        lr_policy="constant",
        lr_min_ratio=0.1,
        lr_max_score=1024,
        lr_lut=(),
    ):
        self.key_dtype = np.dtype(key_dtype)
        self.value_dtype = value_dtype
        self.optimizer_dtype = optimizer_dtype or value_dtype
        self.gradient_dtype = gradient_dtype or value_dtype
        d = np.asarray(dims, dtype=np.int64)
        self._dims = d
        self._lut = np.asarray(lr_lut, dtype=np.float32)
        self._h = lib().or_store_create(
            _ptr(d), len(d), KEY_CODES[self.key_dtype.name], VALUE_CODES[value_dtype],
            VALUE_CODES[self.optimizer_dtype], VALUE_CODES[self.gradient_dtype], gradient_scale,
            int(enable_optimizer), INIT_CODES[init], init_min, init_max,
            OPT_CODES[optimizer if enable_optimizer else "none"], lr, beta1, beta2, eps, weight_decay,
            initial_accumulator, simd_width, threads,
            {"none": 0, "lfu": 1, "lru": 2, "manual": 3}[score_policy],
            {"constant": 0, "sqrt": 1, "log": 2, "inverse": 3, "cosine": 4, "lut": 5}[lr_policy],
            lr_min_ratio, lr_max_score, _ptr(self._lut) if len(self._lut) else None, len(self._lut),
        )

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().or_store_destroy(h)
            self._h = None

    def _vals(self, n, dim, dtype_name):
        if dtype_name == "float32":
            return np.empty(n * dim, dtype=np.float32)
        return np.empty(n * dim, dtype=np.uint16)  # raw f16/bf16 bits

    def reserve(self, n: int, dim: int) -> None:
        _check(lib().or_store_reserve(self._h, dim, n))

    def lookup(self, keys, dim):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        out = self._vals(len(keys), dim, self.value_dtype)
        _check(lib().or_lookup(self._h, _ptr(keys), len(keys), dim, _ptr(out)))
        return out

    def lookup_or_insert(self, keys, dim):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        out = self._vals(len(keys), dim, self.value_dtype)
        _check(lib().or_lookup_or_insert(self._h, _ptr(keys), len(keys), dim, _ptr(out)))
        return out

    def accumulate_gradients(self, keys, grads, dim):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        grads = np.ascontiguousarray(grads)
        _check(lib().or_accumulate_gradients(self._h, _ptr(keys), len(keys), dim, _ptr(grads)))

    def optimizer_step(self, normalization_steps=1):
        _check(lib().or_optimizer_step(self._h, normalization_steps))

    def contains(self, keys):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        out = np.zeros(len(keys), dtype=np.uint8)
        lib().or_contains(self._h, _ptr(keys), len(keys), _ptr(out))
        return out

    def assign(self, keys, values, dim):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        values = np.ascontiguousarray(values)
        _check(lib().or_assign(self._h, _ptr(keys), len(keys), dim, _ptr(values)))

    def erase(self, keys, dim=0):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        _check(lib().or_erase(self._h, _ptr(keys), len(keys), dim))

    def assign_scores(self, keys, scores):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        scores = np.ascontiguousarray(scores, dtype=np.uint64)
        lib().or_assign_scores(self._h, _ptr(keys), len(keys), _ptr(scores))

    def read_scores(self, keys):
        keys = np.ascontiguousarray(keys, dtype=self.key_dtype)
        out = np.zeros(len(keys), dtype=np.uint64)
        lib().or_read_scores(self._h, _ptr(keys), len(keys), _ptr(out))
        return out

    def size(self, dim=0) -> int:
        return int(lib().or_store_size(self._h, dim))

    def dropped(self) -> int:
        return int(lib().or_store_dropped(self._h))

    def read_row(self, key, dim, nstate=0):
        """(found, param[dim], state[nstate*dim], step) of one key, raw dtype bits."""
        p = self._vals(1, dim, self.value_dtype)
        s = self._vals(1, max(nstate, 1) * dim, self.optimizer_dtype)
        step = np.zeros(1, dtype=np.uint32)
        found = lib().or_read_row(self._h, dim, int(np.uint64(np.int64(key)) if key < 0 else key),
                                  _ptr(p), _ptr(s), _ptr(step))
        return bool(found), p, s[: nstate * dim], int(step[0])


def unique_first_occurrence(keys):
    """se::ops::unique_keys_inverse_sequential (sparse_embedding/src/ops/unique_ops.hpp:73-125):
    the distinct keys in order of first appearance (the insertion order of its
    map, which is also the uid each key receives), int32 inverse indices,
    first positions and counts."""
    keys = np.asarray(keys)
    if keys.size == 0:
        e = np.empty(0, dtype=np.int32)
        return keys[:0].copy(), e, e, e
    u, first, inv, counts = np.unique(keys, return_index=True, return_inverse=True, return_counts=True)
    order = np.argsort(first, kind="stable")
    rank = np.empty_like(order)
    rank[order] = np.arange(len(order))
    return (u[order], rank[inv.reshape(-1)].astype(np.int32), first[order].astype(np.int32),
            counts[order].astype(np.int32))


def pool_bags(rows, offsets):
    """Sum pooling of multi-hot bags as the DLRM harness does it (a fixed id
    order per (sample, table)): out[b] = rows[offsets[b]] + rows[offsets[b]+1]
    + ... in float32, one add at a time in key order from +0.0 (numpy's
    reductions may add pairwise, so the adds are stepped by position)."""
    rows = np.asarray(rows, dtype=np.float32)
    offsets = np.asarray(offsets, dtype=np.int64)
    nb = len(offsets) - 1
    lens = np.diff(offsets)
    out = np.zeros((nb, rows.shape[1]), dtype=np.float32)
    for k in range(int(lens.max()) if nb else 0):
        live = np.nonzero(lens > k)[0]
        out[live] = out[live] + rows[offsets[live] + k]
    return out


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
