"""Partition kernels against the reference's golden vectors and the oracle (GPU)."""

import json

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CLS = {"modulo": se.ModuloPartitioner, "hash": se.HashPartitioner, "fast_range": se.FastRangePartitioner}


@pytest.fixture(scope="module")
def vectors(golden_dir):
    return json.loads((golden_dir / "partition_vectors.json").read_text())


def test_golden_cases_bit_exact(vectors):
    for c in vectors["cases"]:
        keys = np.array(c["keys"], dtype=c["key_dtype"])
        p = CLS[c["algorithm"]](num_shards=c["partition_count"])
        got = np.asarray(p.partition(keys))
        assert got.dtype == np.uint32
        np.testing.assert_array_equal(got, np.array(c["partition_ids"], dtype=np.uint32),
                                      err_msg=f'{c["algorithm"]} {c["key_dtype"]} {c["partition_count"]}')
        tgt = c["partition_ids"][-1]
        np.testing.assert_array_equal(np.asarray(p.filter(keys, tgt)), np.array(c["partition_ids"]) == tgt)


def test_modulo_reference_vectors(vectors):
    for v in vectors["modulo_reference_vectors"]:
        keys = np.array([v["logical_key"]], dtype=v["key_dtype"])
        p = se.create_partitioner(se.SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, v["partition_count"])
        assert int(np.asarray(p.partition(keys))[0]) == v["partition_id"]


@pytest.mark.parametrize("dtype", ["int32", "uint32", "int64", "uint64"])
@pytest.mark.parametrize("kind", ["modulo", "hash", "fast_range"])
def test_random_keys_match_oracle(dtype, kind):
    rng = np.random.default_rng(11)
    info = np.iinfo(dtype)
    keys = rng.integers(info.min, info.max, size=1 << 20, dtype=dtype, endpoint=True)
    for n in (1, 2, 3, 7, 8, 13, 64, 1000, 2**32 - 1):
        got = np.asarray(CLS[kind](num_shards=n).partition(keys))
        np.testing.assert_array_equal(got, O.partition(kind, n, keys))


def test_reference_test_ops_cases():
    # sparse_embedding/tests/test_ops.py:155-254 and test_reference_vectors.py
    keys = np.array([10, 11, 12, 13, 14, 15], dtype=np.uint64)
    m = se.ModuloPartitioner(num_shards=2)
    np.testing.assert_array_equal(np.from_dlpack(m.partition(keys)), [0, 1, 0, 1, 0, 1])
    np.testing.assert_array_equal(np.from_dlpack(m.filter(keys, target_shard=0)), [True, False] * 3)
    h = se.HashPartitioner(num_shards=4)
    ids = np.from_dlpack(h.partition(keys))
    np.testing.assert_array_equal(np.from_dlpack(h.filter(keys, target_shard=1)), ids == 1)
    keys = np.asarray([-5, -4, -3, -2, -1, 0, 1, 2, 3], dtype=np.int64)
    for n in (2, 3, 5):
        p = se.ModuloPartitioner(num_shards=n)
        exp = np.mod(keys, np.int64(n)).astype(np.uint32)
        np.testing.assert_array_equal(np.from_dlpack(p.partition(keys)), exp)
        for t in range(n):
            np.testing.assert_array_equal(np.from_dlpack(p.filter(keys, t)), exp == t)
    for dtype, values in ((np.int32, (-5, -1, 0, 1, 5)), (np.uint32, (0, 1, 5, 2**32 - 1)),
                          (np.int64, (-(2**63), -5, -1, 0, 1, 5)), (np.uint64, (0, 1, 5, 2**63 + 1, 2**64 - 1))):
        k = np.asarray(values, dtype=dtype)
        np.testing.assert_array_equal(np.from_dlpack(se.ModuloPartitioner(num_shards=3).partition(k)),
                                      [int(v) % 3 for v in values])
    np.testing.assert_array_equal(
        np.from_dlpack(se.ModuloPartitioner(num_shards=2**32 - 1).partition(np.asarray([-1, 0, 1], np.int32))),
        [2**32 - 2, 0, 1])
    keys = np.arange(100_000, dtype=np.int64) - 50_000
    p = se.ModuloPartitioner(num_shards=16)
    for threads in (0, 1, 2, 4, 8):
        np.testing.assert_array_equal(np.from_dlpack(p.partition(keys, num_threads=threads)),
                                      np.mod(keys, 16).astype(np.uint32))
    k, r = se.generate_reference_vectors(se.SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, key_dtype="int64",
                                         partition_count=5, sample_keys=[10, 25, 42, 99, 100])
    np.testing.assert_array_equal(r, [0, 0, 2, 4, 0])
    for algo in (se.SPARSE_EMBEDDING_MODULO_ASSIGNMENT_NAME, se.SPARSE_EMBEDDING_HASH_ASSIGNMENT_NAME,
                 se.SPARSE_EMBEDDING_FAST_RANGE_ASSIGNMENT_NAME):
        for dt in ["int32", "uint32", "int64", "uint64"]:
            k, r = se.generate_reference_vectors(algo, key_dtype=dt, partition_count=8)
            assert r.dtype == np.uint32 and r.max() < 8
            kind = algo.split(".")[1]
            np.testing.assert_array_equal(r, O.partition(kind, 8, k))


def test_empty_and_cuda_inputs():
    p = se.HashPartitioner(num_shards=8)
    assert np.asarray(p.partition(np.zeros(0, np.int64))).shape == (0,)
    keys = torch.randint(-2**62, 2**62, (300_001,), dtype=torch.int64, device="cuda")
    got = p.partition(keys)
    assert got.is_cuda and got.dtype == torch.uint32
    np.testing.assert_array_equal(got.cpu().numpy(), O.partition("hash", 8, keys.cpu().numpy()))
    mask = p.filter(keys, 3)
    assert mask.is_cuda and mask.dtype == torch.bool
    np.testing.assert_array_equal(mask.cpu().numpy(), got.cpu().numpy() == 3)


@pytest.mark.parametrize("n,parts", [(0, 4), (1, 1), (5000, 3), (65536, 8), (1_000_003, 7)])
def test_route_is_stable_grouping(n, parts):
    rng = np.random.default_rng(n)
    keys_np = rng.integers(-2**63, 2**63 - 1, size=n, dtype=np.int64)
    keys = torch.from_numpy(keys_np).cuda()
    p = se.HashPartitioner(num_shards=parts)
    send_keys, send_pos, counts = p.route(keys)
    torch.cuda.synchronize()
    ids = O.partition("hash", parts, keys_np)
    order = np.argsort(ids, kind="stable")
    np.testing.assert_array_equal(send_pos.cpu().numpy().view(np.uint32), order.astype(np.uint32))
    np.testing.assert_array_equal(send_keys.cpu().numpy(), keys_np[order])
    np.testing.assert_array_equal(counts.cpu().numpy(), np.bincount(ids, minlength=parts))


def test_permute_rows_roundtrip():
    from sparse_embedding_b200 import _native as N

    n, d = 10_000, 64
    rows = torch.randn(n, d, device="cuda")
    perm = torch.randperm(n, device="cuda").to(torch.int32)
    gathered = torch.empty_like(rows)
    back = torch.empty_like(rows)
    st = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().se_permute_rows(rows.data_ptr(), gathered.data_ptr(), perm.data_ptr(), n, d * 4, 1, 0, st))
    N.check(N.lib().se_permute_rows(gathered.data_ptr(), back.data_ptr(), perm.data_ptr(), n, d * 4, 0, 0, st))
    torch.cuda.synchronize()
    assert torch.equal(gathered, rows[perm.long()])
    assert torch.equal(back, rows)
