"""The C++ boundary (include/se_gpu_store.hpp) compiled against libse_gpu.so.

CPU: the header and tests/cpp/gpu_store_test.cpp compile and link with g++
(C++20), so a signature or type mismatch between the C++ types and the C ABI
fails here. GPU: the same program runs the reference-style store test
(normalized SGD in both accumulation modes, lookup semantics, mutation calls,
the reference's exception classes and messages, partition ids)."""

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
LIB_DIR = REPO / "sparse_embedding_b200" / "_lib"
SRC = REPO / "tests" / "cpp" / "gpu_store_test.cpp"


def build_test(out_dir: Path) -> Path:
    assert (LIB_DIR / "libse_gpu.so").exists(), "libse_gpu.so is not built (python -m sparse_embedding_b200.build)"
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = out_dir / "gpu_store_test"
    subprocess.run([gxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I", str(REPO / "include"), str(SRC),
                    "-L", str(LIB_DIR), "-lse_gpu", f"-Wl,-rpath,{LIB_DIR}", "-o", str(exe)], check=True)
    return exe


def test_cpp_boundary_compiles(tmp_path):
    assert build_test(tmp_path).exists()


@pytest.mark.gpu
def test_cpp_boundary_runs(tmp_path):
    exe = build_test(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "gpu_store_test ok" in r.stdout
