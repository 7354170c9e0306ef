"""Array plumbing between user inputs (numpy, torch, DLPack) and the C ABI.

Host arrays are handed to the library as host pointers (it stages them to the
device itself); CUDA tensors are handed over in place together with the
current torch stream of their device.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np

_TORCH = None


def torch_mod():
    global _TORCH
    if _TORCH is None:
        import torch

        _TORCH = torch
    return _TORCH


_NP_NAMES = {
    "int32": "int32", "uint32": "uint32", "int64": "int64", "uint64": "uint64",
    "float32": "float32", "float16": "float16", "bool": "bool", "uint8": "uint8",
}


def _torch_dtype_name(t) -> str:
    name = str(t.dtype).replace("torch.", "")
    return {"float": "float32", "half": "float16", "long": "int64", "int": "int32"}.get(name, name)


def torch_dtype(name: str):
    torch = torch_mod()
    return {
        "int32": torch.int32, "uint32": torch.uint32, "int64": torch.int64, "uint64": torch.uint64,
        "float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
        "uint8": torch.uint8, "bool": torch.bool,
    }[name]


@dataclass
class Arr:
    """A contiguous input array: its pointer, dtype name, shape and memory space."""

    obj: Any
    ptr: int
    dtype: str
    shape: tuple
    cuda_device: int | None  # None for host memory
    stream: int | None       # cudaStream_t of the current torch stream (CUDA inputs)
    is_torch: bool
    pinned: bool = False

    @property
    def size(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n


def is_torch_tensor(x) -> bool:
    if _TORCH is None:
        mod = type(x).__module__
        if not mod.startswith("torch"):
            return False
    torch = torch_mod()
    return isinstance(x, torch.Tensor)


def as_input(x, what: str = "tensor") -> Arr:
    """Wraps x without copying. Raises ValueError when x is not C-contiguous."""
    if is_torch_tensor(x):
        if not x.is_contiguous():
            raise ValueError("tensor must be C-contiguous")
        dev = x.device
        if dev.type == "cuda":
            torch = torch_mod()
            stream = torch.cuda.current_stream(dev).cuda_stream
            return Arr(x, x.data_ptr(), _torch_dtype_name(x), tuple(x.shape), dev.index, stream, True)
        if dev.type != "cpu":
            raise ValueError("only CPU and CUDA tensors are supported")
        return Arr(x, x.data_ptr(), _torch_dtype_name(x), tuple(x.shape), None, None, True, bool(x.is_pinned()))
    if not isinstance(x, np.ndarray):
        if hasattr(x, "__dlpack__"):
            dev = x.__dlpack_device__() if hasattr(x, "__dlpack_device__") else (1, 0)
            if dev[0] != 1:  # not kDLCPU: go through torch, which understands device capsules
                return as_input(torch_mod().from_dlpack(x), what)
            try:
                x = np.from_dlpack(x)
            except (TypeError, RuntimeError, BufferError):
                return as_input(torch_mod().from_dlpack(x), what)
        else:
            x = np.asarray(x)
    if not x.flags.c_contiguous:
        raise ValueError("tensor must be C-contiguous")
    name = _NP_NAMES.get(x.dtype.name, x.dtype.name)
    return Arr(x, x.ctypes.data if x.size else 0, name, tuple(x.shape), None, None, False)


def empty_like_space(ref: Arr, shape, dtype: str):
    """Output array in the memory space of `ref` (numpy for host numpy inputs)."""
    if ref.cuda_device is not None:
        torch = torch_mod()
        return torch.empty(shape, dtype=torch_dtype(dtype), device=f"cuda:{ref.cuda_device}")
    if ref.is_torch or dtype == "bfloat16":
        torch = torch_mod()
        return torch.empty(shape, dtype=torch_dtype(dtype), pin_memory=ref.pinned)
    return np.empty(shape, dtype=np.dtype(dtype))


def data_ptr(a) -> int:
    if isinstance(a, np.ndarray):
        return a.ctypes.data if a.size else 0
    return a.data_ptr()
