"""Embedding bag on the GPU (sum-pooled gather and its backward) against the
oracle (GPU): pooled rows bit-exact with the oracle's rows pooled in key
order; the backward equals accumulate_gradients with each bag's gradient
repeated for its keys (updated rows within the fp32 tolerance of the store
tests)."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_gpu_store import ATOL_FP32, RTOL_FP32, as_float, bits, pair

pytestmark = pytest.mark.gpu


def bags(rng, nbags, mean, pool, dtype):
    lens = rng.poisson(mean, size=nbags)
    lens[rng.random(nbags) < 0.05] = 0  # some empty bags
    offsets = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    keys = rng.choice(pool, size=int(offsets[-1])).astype(dtype)
    return keys, offsets


def expected_pool(orc, keys, offsets, dim, value_dtype, insert):
    raw = orc.lookup_or_insert(keys, dim) if insert else orc.lookup(keys, dim)
    rows = as_float(raw, value_dtype).reshape(-1, dim)
    pooled = O.pool_bags(rows, offsets)
    if value_dtype == "float32":
        return pooled.view(np.uint32)
    if value_dtype == "float16":
        return pooled.astype(np.float16).view(np.uint16)
    return np.vectorize(O.lib().or_f32_to_bf16, otypes=[np.uint16])(pooled)


@pytest.mark.parametrize("value_dtype,dim", [("float32", 128), ("bfloat16", 24), ("float16", 7), ("float32", 64)])
def test_pool_matches_the_oracle(value_dtype, dim):
    rng = np.random.default_rng(dim)
    gpu, orc = pair([dim], key_dtype="int64", value_dtype=value_dtype, opt="adam")
    pool = rng.integers(-2**63, 2**63 - 1, size=20_000, dtype=np.int64)
    keys, offsets = bags(rng, 3000, 12, pool, np.int64)
    got = gpu.embedding_bag(keys, offsets, dim, insert=True)
    np.testing.assert_array_equal(bits(got).reshape(len(offsets) - 1, dim),
                                  expected_pool(orc, keys, offsets, dim, value_dtype, True))
    # without insert: keys never seen add zero rows
    k2, o2 = bags(rng, 2000, 8, np.concatenate([pool[:5000], rng.integers(0, 2**40, size=5000)]), np.int64)
    got = gpu.embedding_bag(torch.from_numpy(k2).cuda(), torch.from_numpy(o2).cuda(), dim, insert=False)
    assert got.is_cuda
    np.testing.assert_array_equal(bits(got).reshape(len(o2) - 1, dim),
                                  expected_pool(orc, k2, o2, dim, value_dtype, False))
    assert gpu.total_size() == orc.size()


def test_backward_equals_repeated_gradients_and_trains_like_the_oracle():
    rng = np.random.default_rng(11)
    dim = 128
    gpu, orc = pair([dim], key_dtype="uint64", opt="adam", lr=1e-3)
    pool = rng.integers(0, 2**64 - 1, size=30_000, dtype=np.uint64)
    for step in range(3):
        keys, offsets = bags(rng, 4096, 20, pool, np.uint64)
        gpu.embedding_bag(keys, offsets, dim)
        orc.lookup_or_insert(keys, dim)
        g = (rng.standard_normal((len(offsets) - 1, dim)) * 1e-3).astype(np.float32)
        gpu.embedding_bag_backward(keys, offsets, g)
        bag_of = np.repeat(np.arange(len(offsets) - 1), np.diff(offsets))
        orc.accumulate_gradients(keys, g[bag_of], dim)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    probe = np.unique(pool)
    got, _ = gpu.lookup(probe, dim)
    np.testing.assert_allclose(np.asarray(got).reshape(-1, dim), orc.lookup(probe, dim).reshape(-1, dim),
                               rtol=RTOL_FP32, atol=ATOL_FP32)


def test_autograd_wrapper_matches_the_explicit_backward():
    from sparse_embedding_b200.torch_ops import embedding_bag

    rng = np.random.default_rng(12)
    dim = 64
    a, _ = pair([dim], key_dtype="int64", opt="sgd", lr=0.1)
    b, _ = pair([dim], key_dtype="int64", opt="sgd", lr=0.1)
    keys, offsets = bags(rng, 1024, 6, np.arange(5000, dtype=np.int64), np.int64)
    k, o = torch.from_numpy(keys).cuda(), torch.from_numpy(offsets).cuda()
    w = torch.randn((len(offsets) - 1, dim), device="cuda")
    pooled = embedding_bag(a, k, o, dim)
    (pooled * w).sum().backward()
    b.embedding_bag(k, o, dim)
    b.embedding_bag_backward(k, o, w)
    a.optimizer_step(1)
    b.optimizer_step(1)
    probe = np.arange(5000, dtype=np.int64)
    np.testing.assert_array_equal(bits(a.lookup(probe, dim)[0]), bits(b.lookup(probe, dim)[0]))


def test_offset_checks():
    gpu, _ = pair([8], opt="sgd")
    keys = np.arange(6, dtype=np.int64)
    with pytest.raises(ValueError, match="start at 0"):
        gpu.embedding_bag(keys, np.array([1, 3, 6], dtype=np.int64), 8)
    with pytest.raises(ValueError, match="non-decreasing"):
        gpu.embedding_bag(keys, np.array([0, 4, 3, 6], dtype=np.int64), 8)
    with pytest.raises(ValueError, match="int64"):
        gpu.embedding_bag(keys, np.array([0, 6], dtype=np.int32), 8)
    out = gpu.embedding_bag(keys, np.array([0, 0, 6, 6], dtype=np.int64), 8)
    assert np.asarray(out).shape == (3, 8) and not np.asarray(out)[0].any() and not np.asarray(out)[2].any()
