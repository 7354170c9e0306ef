"""GPU unique (se_unique) against the oracle's restatement of the reference's
sequential unique_keys_inverse: identical outputs, element for element
(distinct keys in order of first appearance, inverse indices, first
positions, counts), plus the reference's own cases (tests/test_ops.py:9-153) (GPU)."""

import asyncio

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [np.int32, np.uint32, np.int64, np.uint64]


def host(x):
    return x.cpu().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)


def check_against_oracle(keys, res):
    u, inv, first, counts = (host(r) for r in res)
    ru, rinv, rfirst, rcounts = O.unique_first_occurrence(host(keys))
    np.testing.assert_array_equal(u, ru)
    np.testing.assert_array_equal(inv, rinv)
    np.testing.assert_array_equal(first, rfirst)
    np.testing.assert_array_equal(counts, rcounts)
    assert inv.dtype == first.dtype == counts.dtype == np.int32 and u.dtype == host(keys).dtype


def test_reference_cases():
    keys = np.array([10, 20, 10, 30, 20, 40], dtype=np.int64)

    async def run(**kw):
        return await se.async_unique(keys, **kw)

    u, inv = asyncio.run(run())
    np.testing.assert_array_equal(u[inv], keys)
    check_against_oracle(keys, asyncio.run(run(return_first_indices=True, return_counts=True)))
    k32 = np.array([10, 20, 10, 30], dtype=np.int32)
    u, first, counts = se.unique(k32, return_inverse=False, return_first_indices=True, return_counts=True)
    assert u.tolist() == [10, 20, 30] and first.tolist() == [0, 1, 3] and counts.tolist() == [2, 1, 1]


@pytest.mark.parametrize("dtype", DTYPES)
def test_random_and_boundary_keys_match_the_oracle(dtype):
    rng = np.random.default_rng(42)
    info = np.iinfo(dtype)
    edge = np.array([info.min, info.max, 0, 1, info.max - 1], dtype=dtype)  # int64 -1 / uint64 max: the all-ones key
    if np.issubdtype(dtype, np.signedinteger):
        edge = np.concatenate([edge, np.array([-1, -2], dtype=dtype)])
    for n in (1, 7, 5000, 50_000, 1_000_003):
        keys = rng.integers(0, max(2, n // 3), size=n, dtype=np.int64).astype(dtype)
        keys[rng.integers(0, n, size=min(n, 20))] = rng.choice(edge, size=min(n, 20))
        check_against_oracle(keys, se.unique(keys, return_first_indices=True, return_counts=True))
    # device tensors stay on the device
    keys = torch.from_numpy(keys.view(np.int64) if dtype == np.uint64 else keys).cuda()
    if dtype == np.uint64:
        keys = keys.view(torch.uint64)
    res = se.unique(keys, return_first_indices=True, return_counts=True)
    assert all(r.is_cuda for r in res)
    check_against_oracle(keys, res)


def test_zipf_batches_and_repeated_calls():
    from sparse_embedding_b200.workloads import TrainWorkload

    wl = TrainWorkload(num_keys=1_000_000, batch=65_536)
    keys, _ = wl.make_batches(3)
    for b in keys:
        check_against_oracle(b, se.unique(b, return_first_indices=True, return_counts=True))
        d = torch.from_numpy(b).cuda()
        check_against_oracle(d, se.unique(d, return_first_indices=True, return_counts=True))


@pytest.mark.parametrize("keys", [np.array([[1, 2]], dtype=np.int64), np.arange(10, dtype=np.int64)[::2]])
def test_rejects_unsupported_layout(keys):
    with pytest.raises(ValueError):
        se.async_unique(keys)


@pytest.mark.parametrize("dtype", DTYPES)
def test_empty_and_singleton(dtype):
    async def run(k):
        return await se.async_unique(k, return_first_indices=True, return_counts=True, num_threads=2)

    for out in asyncio.run(run(np.empty(0, dtype=dtype))):
        assert np.asarray(out).size == 0
    keys = np.arange(2, dtype=dtype)[::2]
    assert keys.flags.c_contiguous
    u, inv = se.unique(keys)
    np.testing.assert_array_equal(u[inv], keys)


def test_optional_outputs_through_the_c_abi():
    import ctypes as C

    from sparse_embedding_b200 import _native as N

    keys = torch.tensor([5, 5, 9, 5, 2], dtype=torch.int64, device="cuda")
    u = torch.empty(5, dtype=torch.int64, device="cuda")
    counts = torch.empty(5, dtype=torch.int32, device="cuda")
    cnt = C.c_uint64()
    N.check(N.lib().se_unique(N.KEY_CODES["int64"], keys.data_ptr(), 5, u.data_ptr(), None, None,
                              counts.data_ptr(), C.byref(cnt), 0, None))
    assert cnt.value == 3 and u[:3].tolist() == [5, 9, 2] and counts[:3].tolist() == [3, 1, 1]
