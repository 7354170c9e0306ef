"""Checkpoint interop of the GPU store with the reference's Python API
(sparse_embedding/src/bindings/module.cpp:776-805,
bindings/typed/module_typed_checkpoint.inl:146-200): export of every table's
present keys with their rows (and optimizer state) in batches handed to a
visitor, and assign_opt_state to load optimizer state back. Together with
EmbeddingStore.assign this moves a store's contents through host memory,
e.g. to and from the reference's Lance checkpoints.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N


def _np_dtype(name: str):
    return np.uint16 if name in ("bfloat16", "float16") else np.dtype(name)


def _raw_to_array(raw: np.ndarray, name: str):
    if name == "float16":
        return raw.view(np.float16)
    if name == "bfloat16":
        from ._tensors import torch_mod

        return torch_mod().from_numpy(raw.view(np.int16)).view(torch_mod().bfloat16)
    return raw


def _state_count(store) -> int:
    if not store.optimizer_enabled():
        return 0
    return {"adam": 2, "adagrad": 1}.get(getattr(store._optimizer, "kind", ""), 0)


def export_batches(store, batch_size: int = 65536, include_optimizer_state: bool = False,
                   include_steps: bool = False):
    """Yields (dim, keys, values[, opt_states][, steps]) per batch of at most
    batch_size present keys of each table; host arrays, values [n, dim]."""
    if int(batch_size) <= 0:
        raise ValueError("batch_size must be > 0")
    lib = N.lib()
    ns = _state_count(store)
    for dim in store.table_dims():
        total = C.c_uint64()
        N.check(lib.se_export_snapshot(store._h, int(dim), C.byref(total), None))
        for off in range(0, int(total.value), int(batch_size)):
            n = min(int(batch_size), int(total.value) - off)
            keys = np.empty(n, dtype=np.dtype(store.key_dtype()))
            vals = np.empty((n, dim), dtype=_np_dtype(store.value_dtype()))
            states = np.empty((n, ns * dim), dtype=_np_dtype(store.optimizer_dtype())) \
                if include_optimizer_state and ns else None
            steps = np.empty(n, dtype=np.uint32) if include_steps else None
            N.check(lib.se_export_read(store._h, int(dim), off, n, keys.ctypes.data, vals.ctypes.data,
                                       states.ctypes.data if states is not None else None,
                                       steps.ctypes.data if steps is not None else None, None))
            out = [int(dim), keys, _raw_to_array(vals, store.value_dtype())]
            if include_optimizer_state:
                out.append(_raw_to_array(states, store.optimizer_dtype()) if states is not None
                           else np.empty((n, 0), dtype=np.float32))
            if include_steps:
                out.append(steps)
            yield tuple(out)


def export_batches_dlpack(store, visitor, batch_size: int = 65536, include_optimizer_state: bool = False) -> None:
    """The reference's visitor form: visitor(dim, keys, values[, opt_states])
    for each batch (module_typed_checkpoint.inl:146-200)."""
    for batch in export_batches(store, batch_size, include_optimizer_state):
        visitor(*batch)


def assign_opt_state(store, keys, opt_states, dimension: int, steps=None) -> None:
    """Sets the optimizer state rows (and Adam steps) of present keys
    (assign_opt_states, hogwild_embedding_store.hpp:6278-6351)."""
    from ._tensors import as_input

    k = store._keys(keys)
    s = as_input(opt_states, "opt_states")
    if s.dtype != store.optimizer_dtype():
        raise ValueError("dtype mismatch in dlpack_to_span")
    st = None
    if steps is not None:
        st = as_input(steps, "steps")
        if st.dtype != "uint32" or st.size != k.size:
            raise ValueError("assign_opt_states step count does not match key count")
    if (k.cuda_device is None) != (s.cuda_device is None):
        raise ValueError("keys and opt_states must be in the same memory space")
    N.check(N.lib().se_assign_opt_states(store._h, int(dimension), k.ptr, k.size, s.ptr, s.size,
                                         st.ptr if st is not None else None, store._stream(k)))
