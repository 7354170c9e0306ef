"""Generates the golden fixtures in this folder from the reference itself.

Run in a checkout that has the reference sources (default: the checkout named
"reference" beside this repository) and
the reference shim built (`make -C oracle ref`, which compiles the reference's
own ops/partitioner.hpp and simd/*_ops.hpp in place):

    python tests/golden/make_golden.py [REF_ROOT]

Outputs:
  partition_vectors.json  - the reference's modulo reference vectors
                            (sparse_embedding/tests/data/modulo_assignment_reference_vectors.json),
                            re-checked against the compiled reference partitioner,
                            plus hash / fast_range / modulo ids of boundary and
                            random keys for every key dtype, computed by the
                            compiled reference partitioners.
  row_math.npz            - simd_uniform_init rows (f32, bf16, f16) and
                            simd_sgd_update / simd_adam_update results, computed
                            by the compiled reference kernels.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import oracle as O  # noqa: E402

COUNTS = [1, 2, 3, 5, 7, 8, 16, 1000, 2**31, 2**32 - 1]
KINDS = ["modulo", "hash", "fast_range"]


def boundary_keys(dtype: str) -> list[int]:
    info = np.iinfo(dtype)
    ks = {int(info.min), int(info.max), 0, 1, 2, 3, 1024, 1048576, (1 << 30) - 1}
    if info.min < 0:
        ks |= {-1, -2, -3, -1024, -1048576, -(1 << 30), int(info.min) + 1}
    else:
        ks |= {1 << (info.bits - 1), (1 << 31) - 1, int(info.max) - 1}
    return sorted(ks)


def main(ref_root: str) -> None:
    ref_json = Path(ref_root) / "sparse_embedding/tests/data/modulo_assignment_reference_vectors.json"
    reference = json.loads(ref_json.read_text())
    # The reference's own vectors must agree with its compiled partitioner.
    for v in reference["vectors"]:
        keys = np.array([v["logical_key"]], dtype=v["key_dtype"])
        got = int(O.ref_partition("modulo", v["partition_count"], keys)[0])
        assert got == v["partition_id"], v

    rng = np.random.default_rng(20261201)
    cases = []
    for dtype in ["int32", "uint32", "int64", "uint64"]:
        info = np.iinfo(dtype)
        rand = rng.integers(info.min, info.max, size=48, dtype=dtype, endpoint=True)
        keys = np.concatenate([np.array(boundary_keys(dtype), dtype=dtype), rand])
        for kind in KINDS:
            for count in COUNTS:
                ids = O.ref_partition(kind, count, keys)
                cases.append({
                    "algorithm": kind, "key_dtype": dtype, "partition_count": count,
                    "keys": [int(k) for k in keys], "partition_ids": [int(i) for i in ids],
                })
    out = {
        "source": "compiled reference ops/partitioner.hpp via oracle/_ref",
        "modulo_reference_vectors": reference["vectors"],
        "cases": cases,
    }
    (HERE / "partition_vectors.json").write_text(json.dumps(out, separators=(",", ":")))

    R = O.ref()
    init_keys = np.array([0, 1, 2, 12345, 2**32 - 1, 2**32, 2**63, 2**64 - 1, 0xDEADBEEFCAFEF00D], dtype=np.uint64)
    init_dims = np.array([1, 3, 8, 16, 17, 32, 64, 100, 128, 256], dtype=np.int64)
    f32 = np.zeros((len(init_keys), len(init_dims), 256), dtype=np.float32)
    bf = np.zeros((len(init_keys), len(init_dims), 256), dtype=np.uint16)
    hf = np.zeros((len(init_keys), len(init_dims), 256), dtype=np.uint16)
    for a, key in enumerate(init_keys):
        for b, dim in enumerate(init_dims):
            R.ref_uniform_init_f32(f32[a, b].ctypes.data, int(dim), -0.05, 0.05, int(key))
            R.ref_uniform_init_bf16(bf[a, b].ctypes.data, int(dim), -0.05, 0.05, int(key))
            R.ref_uniform_init_f16(hf[a, b].ctypes.data, int(dim), -0.05, 0.05, int(key))

    opt_dims = np.array([1, 8, 17, 32, 64, 100], dtype=np.int64)
    D = 128
    p0 = rng.standard_normal((len(opt_dims), D)).astype(np.float32) * np.float32(0.05)
    g0 = rng.standard_normal((len(opt_dims), D)).astype(np.float32) * np.float32(0.01)
    m0 = rng.standard_normal((len(opt_dims), D)).astype(np.float32) * np.float32(0.01)
    v0 = np.abs(rng.standard_normal((len(opt_dims), D)).astype(np.float32)) * np.float32(1e-4)
    sgd_out = np.zeros((2, len(opt_dims), D), dtype=np.float32)
    adam_p = np.zeros((2, len(opt_dims), D), dtype=np.float32)
    adam_m = np.zeros_like(adam_p)
    adam_v = np.zeros_like(adam_p)
    for w, wd in enumerate([0.0, 0.01]):
        for b, dim in enumerate(opt_dims):
            p = p0[b].copy()
            R.ref_sgd_f32(p.ctypes.data, g0[b].ctypes.data, 0.01, wd, int(dim))
            sgd_out[w, b] = p
            p, m, v = p0[b].copy(), m0[b].copy(), v0[b].copy()
            R.ref_adam_f32(p.ctypes.data, g0[b].ctypes.data, m.ctypes.data, v.ctypes.data, 1e-3, 0.9, 0.999,
                           1e-8, 10.0, 1000.0, wd, int(dim))
            adam_p[w, b], adam_m[w, b], adam_v[w, b] = p, m, v
    np.savez_compressed(
        HERE / "row_math.npz", init_keys=init_keys, init_dims=init_dims, init_f32=f32, init_bf16=bf,
        init_f16=hf, opt_dims=opt_dims, p0=p0, g0=g0, m0=m0, v0=v0, sgd_out=sgd_out, adam_p=adam_p,
        adam_m=adam_m, adam_v=adam_v, simd_width=np.int64(R.ref_simd_width()),
    )
    print("wrote", HERE / "partition_vectors.json", HERE / "row_math.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(HERE.parents[2] / "reference"))
