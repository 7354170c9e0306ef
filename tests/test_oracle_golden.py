"""The oracle against the reference's own outputs (CPU only).

Pins the restatement in oracle/se_oracle.cpp against the golden fixtures made
from the reference's compiled code (tests/golden/make_golden.py), and, when
oracle/_ref was built here, directly against the compiled reference.
"""

import json

import numpy as np
import pytest

from oracle import oracle as O


@pytest.fixture(scope="module")
def vectors(golden_dir):
    return json.loads((golden_dir / "partition_vectors.json").read_text())


@pytest.fixture(scope="module")
def rowmath(golden_dir):
    return np.load(golden_dir / "row_math.npz")


def test_modulo_reference_vectors(vectors):
    # sparse_embedding/tests/test_key_partition.py:17-80 contract: counts 3 and 7, four dtypes.
    groups = {(v["key_dtype"], v["partition_count"]) for v in vectors["modulo_reference_vectors"]}
    assert groups == {(d, c) for d in ["int32", "uint32", "int64", "uint64"] for c in (3, 7)}
    for v in vectors["modulo_reference_vectors"]:
        keys = np.array([v["logical_key"]], dtype=v["key_dtype"])
        assert v["logical_key"] % v["partition_count"] == v["partition_id"]
        assert O.partition("modulo", v["partition_count"], keys)[0] == v["partition_id"]


def test_partition_cases_match_compiled_reference(vectors):
    assert len(vectors["cases"]) == 4 * 3 * 10
    for c in vectors["cases"]:
        keys = np.array(c["keys"], dtype=c["key_dtype"])
        got = O.partition(c["algorithm"], c["partition_count"], keys)
        np.testing.assert_array_equal(got, np.array(c["partition_ids"], dtype=np.uint32), err_msg=str(c["algorithm"]))
        tgt = c["partition_ids"][0]
        np.testing.assert_array_equal(O.filter_mask(c["algorithm"], c["partition_count"], keys, tgt),
                                      np.array(c["partition_ids"]) == tgt)


def test_reference_test_ops_cases():
    # sparse_embedding/tests/test_ops.py:155-254
    keys = np.array([10, 11, 12, 13, 14, 15], dtype=np.uint64)
    np.testing.assert_array_equal(O.partition("modulo", 2, keys), [0, 1, 0, 1, 0, 1])
    keys = np.asarray([-5, -4, -3, -2, -1, 0, 1, 2, 3], dtype=np.int64)
    for n in (2, 3, 5):
        np.testing.assert_array_equal(O.partition("modulo", n, keys), np.mod(keys, n).astype(np.uint32))
    np.testing.assert_array_equal(O.partition("modulo", 2**32 - 1, np.asarray([-1, 0, 1], dtype=np.int32)),
                                  [2**32 - 2, 0, 1])
    keys = np.arange(100_000, dtype=np.int64) - 50_000
    np.testing.assert_array_equal(O.partition("modulo", 16, keys), np.mod(keys, 16).astype(np.uint32))
    # test_reference_vectors.py:36-45
    np.testing.assert_array_equal(O.partition("modulo", 5, np.array([10, 25, 42, 99, 100], dtype=np.int64)),
                                  [0, 0, 2, 4, 0])


def test_uniform_init_matches_reference_rows(rowmath):
    for a, key in enumerate(rowmath["init_keys"]):
        for b, dim in enumerate(rowmath["init_dims"]):
            dim = int(dim)
            row = O.uniform_init(dim, int(key))
            np.testing.assert_array_equal(row.view(np.uint32), rowmath["init_f32"][a, b, :dim].view(np.uint32))
            np.testing.assert_array_equal(O.f32_to_bf16_bits(row), rowmath["init_bf16"][a, b, :dim])
            np.testing.assert_array_equal(O.f32_to_f16_bits(row), rowmath["init_f16"][a, b, :dim])


def test_sgd_adam_match_reference_kernels(rowmath):
    L = O.lib()
    for w, wd in enumerate([0.0, 0.01]):
        for b, dim in enumerate(rowmath["opt_dims"]):
            dim = int(dim)
            p = rowmath["p0"][b].copy()
            g = rowmath["g0"][b].copy()
            L.or_sgd_f32(p.ctypes.data, g.ctypes.data, 0.01, wd, dim, 16)
            np.testing.assert_array_equal(p.view(np.uint32), rowmath["sgd_out"][w, b].view(np.uint32))
            p, m, v = rowmath["p0"][b].copy(), rowmath["m0"][b].copy(), rowmath["v0"][b].copy()
            L.or_adam_f32(p.ctypes.data, g.ctypes.data, m.ctypes.data, v.ctypes.data, 1e-3, 0.9, 0.999, 1e-8,
                          10.0, 1000.0, wd, dim, 16)
            np.testing.assert_array_equal(p.view(np.uint32), rowmath["adam_p"][w, b].view(np.uint32))
            np.testing.assert_array_equal(m.view(np.uint32), rowmath["adam_m"][w, b].view(np.uint32))
            np.testing.assert_array_equal(v.view(np.uint32), rowmath["adam_v"][w, b].view(np.uint32))


@pytest.mark.skipif(not O.ref_available(), reason="reference shim (oracle/_ref) not built here")
def test_oracle_matches_compiled_reference_random():
    rng = np.random.default_rng(7)
    for dt in ["int32", "uint32", "int64", "uint64"]:
        info = np.iinfo(dt)
        keys = rng.integers(info.min, info.max, size=20000, dtype=dt, endpoint=True)
        for kind in ["modulo", "hash", "fast_range"]:
            for n in [1, 3, 4, 6, 8, 12, 2**20 + 7]:
                np.testing.assert_array_equal(O.partition(kind, n, keys), O.ref_partition(kind, n, keys))


def test_store_flow_reference_semantics():
    # hogwild_storage_test.cpp:42-103: SGD, N=2 -> value == -lr * 1/2 per element.
    s = O.OracleStore([8], key_dtype="int64", init="zeros", optimizer="sgd", lr=1.0)
    keys = np.arange(4096, dtype=np.int64)
    s.lookup_or_insert(keys, 8)
    g = np.ones((4096, 8), dtype=np.float32)
    s.accumulate_gradients(keys, g, 8)
    s.optimizer_step(2)
    np.testing.assert_allclose(s.lookup(keys, 8), -0.5, atol=1e-6)
    # test_mixed_precision.py:408-438: optimizer_step(N) averages N accumulations -> -3.0.
    s = O.OracleStore([1], key_dtype="int64", init="zeros", optimizer="sgd", lr=1.0, gradient_dtype="float16",
                      gradient_scale=8.0)
    k = np.array([17], dtype=np.int64)
    s.lookup_or_insert(k, 1)
    for _ in range(3):
        s.accumulate_gradients(k, np.array([[3.0]], dtype=np.float16), 1)
    s.optimizer_step(3)
    np.testing.assert_allclose(s.lookup(k, 1), [-3.0], atol=2e-3)
    # Absent keys are dropped at step time.
    s = O.OracleStore([4], key_dtype="uint64", init="zeros", optimizer="sgd", lr=0.1)
    s.accumulate_gradients(np.array([5], dtype=np.uint64), np.ones((1, 4), np.float32), 4)
    s.optimizer_step(1)
    assert s.dropped() == 1 and s.size() == 0


def test_threaded_oracle_matches_serial():
    """The multi-threaded oracle (the timed CPU baseline) computes exactly what
    the serial one does: per key the summation order is the batch order."""
    from sparse_embedding_b200.workloads import TrainWorkload

    wl = TrainWorkload(num_keys=20_000, batch=8192)
    keys, grads = wl.make_batches(3)
    outs = []
    for threads in (1, 4):
        s = O.OracleStore([64], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8,
                          initial_accumulator=0.1, threads=threads)
        s.lookup_or_insert(wl.warm_keys(), 64)
        for b in range(3):
            s.lookup_or_insert(keys[b], 64)
            s.accumulate_gradients(keys[b], grads[b], 64)
            s.optimizer_step(1)
        outs.append(s.lookup(np.unique(keys), 64))
    np.testing.assert_array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_unique_oracle_reference_cases():
    """The oracle's unique against the reference's own cases (tests/test_ops.py:9-153):
    exact reconstruction, first positions, counts, all four key dtypes, empty input."""
    keys = np.array([10, 20, 10, 30, 20, 40], dtype=np.int64)
    u, inv, first, counts = O.unique_first_occurrence(keys)
    assert u.tolist() == [10, 20, 30, 40] and inv.tolist() == [0, 1, 0, 2, 1, 3]
    assert first.tolist() == [0, 1, 3, 5] and counts.tolist() == [2, 2, 1, 1]
    np.random.seed(42)
    for dtype in [np.int32, np.uint32, np.int64, np.uint64]:
        keys = np.random.randint(0, 5000, size=50000, dtype=dtype)
        u, inv, first, counts = O.unique_first_occurrence(keys)
        np.testing.assert_array_equal(u[inv], keys)
        ek, ef, ec = np.unique(keys, return_index=True, return_counts=True)
        np.testing.assert_array_equal(np.sort(u), ek)
        pos = np.searchsorted(ek, u)
        np.testing.assert_array_equal(first, ef[pos])
        np.testing.assert_array_equal(counts, ec[pos])
        assert (np.diff(first) > 0).all()  # order of first appearance
        e = O.unique_first_occurrence(np.empty(0, dtype=dtype))
        assert all(x.size == 0 for x in e)


@pytest.mark.parametrize(
    ("policy", "kw", "score", "expected"),
    [
        ("constant", {}, 37, 1.0),
        ("sqrt", {}, 0, 1.0),
        ("sqrt", {}, 4, 0.5),
        ("log", {}, 2, 0.5),
        ("inverse", {}, 0, 1.0),
        ("inverse", {}, 4, 0.25),
        ("cosine", {"lr_min_ratio": 0.2, "lr_max_score": 4}, 0, 1.0),
        ("cosine", {"lr_min_ratio": 0.2, "lr_max_score": 4}, 2, 0.6),
        ("cosine", {"lr_min_ratio": 0.2, "lr_max_score": 4}, 4, 0.2),
        ("cosine", {"lr_min_ratio": 0.2, "lr_max_score": 4}, 5, 0.2),
        ("lut", {"lr_lut": [0.25, 0.5, 0.75]}, 0, 0.25),
        ("lut", {"lr_lut": [0.25, 0.5, 0.75]}, 2, 0.75),
        ("lut", {"lr_lut": [0.25, 0.5, 0.75]}, 3, 0.75),
    ],
)
def test_oracle_lr_policies_reference_answers(policy, kw, score, expected):
    """The reference's known answers for its policies (tests/test_dynamic_lr.py:35-52):
    an SGD step of lr 1 on a zero row with gradient 1 moves it by -lr(score)."""
    orc = O.OracleStore([16], key_dtype="int64", init="zeros", optimizer="sgd", lr=1.0, score_policy="manual",
                        lr_policy=policy, **kw)
    keys = np.array([7], dtype=np.int64)
    orc.lookup_or_insert(keys, 16)
    orc.assign_scores(keys, np.array([score], dtype=np.uint64))
    orc.accumulate_gradients(keys, np.ones((1, 16), dtype=np.float32), 16)
    orc.optimizer_step(1)
    np.testing.assert_allclose(-orc.lookup(keys, 16), expected, atol=1e-6)


def test_oracle_lfu_lru_scores():
    """LFU counts every found position of a lookup; LRU stamps them with the
    store's clock (from 1) in batch order; lookup_or_insert does not touch."""
    for policy, expect in (("lfu", [3, 1, 0]), ("lru", [4, 2, 0])):
        orc = O.OracleStore([4], key_dtype="int64", optimizer="sgd", score_policy=policy)
        orc.lookup_or_insert(np.array([1, 2, 3], dtype=np.int64), 4)
        orc.lookup(np.array([1, 2, 9, 1], dtype=np.int64), 4)   # 9 is absent
        orc.lookup(np.array([1], dtype=np.int64), 4)
        assert orc.read_scores(np.array([1, 2, 3], dtype=np.int64)).tolist() == expect
