"""The C ABI library loads and exports every entry point include/se_gpu.h declares (CPU only)."""

import ctypes
import re

from sparse_embedding_b200 import _native as N
from sparse_embedding_b200.build import LIB_PATH


def declared_functions(repo):
    text = (repo / "include" / "se_gpu.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\s*\*|uint64_t)\s*(se_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    from tests.conftest import REPO

    names = declared_functions(REPO)
    assert "se_forward_lookup" in names and "se_optimizer_step" in names and len(names) >= 25


def test_library_exports_every_declared_symbol():
    from tests.conftest import REPO

    assert LIB_PATH.exists(), "libse_gpu.so must be built (python -m sparse_embedding_b200.build)"
    lib = ctypes.CDLL(str(LIB_PATH))
    for name in declared_functions(REPO):
        assert hasattr(lib, name), name
        assert name in N.exported_symbols(), f"{name} missing from the ctypes binding"


def test_binding_loads_without_gpu():
    L = N.lib()
    assert L.se_version().startswith(b"se_gpu")
    assert isinstance(L.se_kernel_launch_count(), int)
    # Argument errors are reported before any device work.
    assert L.se_partition(0, 0, 2, None, 0, None, 0, None) == N.SE_ERR_INVALID_ARGUMENT
    assert b"num_shards must be > 0" in L.se_last_error()
    assert L.se_store_create(None, None) == N.SE_ERR_INVALID_ARGUMENT
