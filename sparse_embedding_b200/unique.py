"""Distinct keys with inverse indices, first indices and counts on the GPU
(se_unique), with the contract of the reference's async_unique
(sparse_embedding/src/bindings/module.cpp:959-1072):

- unique_keys: the distinct keys (here in order of first appearance; the
  reference leaves the order unspecified);
- inverse_indices: int32, unique_keys[inverse_indices[i]] == keys[i];
- first_indices: int32, position of the first appearance of each unique key;
- counts: int32, number of appearances of each unique key.

Host inputs give numpy outputs, CUDA tensors give CUDA tensors on the same
device. num_threads is accepted for compatibility and has no effect.
"""

from __future__ import annotations

import asyncio
import ctypes as C

from . import _native as N
from ._tensors import Arr, as_input, data_ptr, empty_like_space
from .partitioner import _device_for


def _keys(keys) -> Arr:
    k = as_input(keys, "keys")
    if len(k.shape) != 1:
        raise ValueError("async_unique requires a 1D tensor")
    if k.dtype not in N.KEY_CODES:
        raise ValueError(f"unsupported key dtype: {k.dtype}")
    if k.size > 0x7FFFFFFF:
        raise ValueError("Input size exceeds maximum supported 32-bit element count (2^31 - 1)")
    return k


def _run(k: Arr, return_inverse: bool, return_first_indices: bool, return_counts: bool) -> tuple:
    n = k.size
    uniq = empty_like_space(k, (n,), k.dtype)
    inv = empty_like_space(k, (n,), "int32") if return_inverse else None
    first = empty_like_space(k, (n,), "int32") if return_first_indices else None
    counts = empty_like_space(k, (n,), "int32") if return_counts else None
    u = 0
    if n:
        cnt = C.c_uint64()
        N.check(N.lib().se_unique(N.KEY_CODES[k.dtype], k.ptr, n, data_ptr(uniq),
                                  data_ptr(inv) if inv is not None else None,
                                  data_ptr(first) if first is not None else None,
                                  data_ptr(counts) if counts is not None else None,
                                  C.byref(cnt), _device_for(k), k.stream))
        u = int(cnt.value)
    out = [uniq[:u]]
    if inv is not None:
        out.append(inv)
    if first is not None:
        out.append(first[:u])
    if counts is not None:
        out.append(counts[:u])
    return tuple(out)


def unique(keys, return_inverse: bool = True, return_first_indices: bool = False, return_counts: bool = False,
           num_threads: int = 0) -> tuple:
    """(unique_keys[, inverse_indices][, first_indices][, counts]) of a 1D key array."""
    del num_threads
    return _run(_keys(keys), return_inverse, return_first_indices, return_counts)


def async_unique(keys, return_inverse: bool = True, return_first_indices: bool = False,
                 return_counts: bool = False, num_threads: int = 0):
    """Awaitable form of unique(); argument errors raise here, before anything runs."""
    del num_threads
    k = _keys(keys)
    return asyncio.to_thread(_run, k, return_inverse, return_first_indices, return_counts)
