"""asyncio variants and clear() of the GPU store (GPU).

Mirrors the reference's test_embedding_table_async
(sparse_embedding/tests/test_embedding_table.py:225-275) and compares every
awaited result with the synchronous call on a twin store."""

import asyncio

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se

pytestmark = pytest.mark.gpu


def make_store():
    return se.EmbeddingStore(se.EmbeddingConfig(dims=[128], thread_budget=4, value_dtype="float32"),
                             initializer_config=se.Zeros(), score_policy="lru")


def test_async_methods_match_sync():
    keys = np.array([1, 2, 3], dtype=np.int64)
    rng = np.random.default_rng(0)
    values = rng.random((3, 128)).astype(np.float32)
    grads = rng.random((3, 128)).astype(np.float32)
    scores = np.array([10, 20, 30], dtype=np.uint64)
    store, twin = make_store(), make_store()

    async def run():
        await store.async_assign(keys, values)
        vals, lens = await store.async_lookup(keys, dim=128)
        assert np.asarray(vals).shape[0] == 3 * 128
        np.testing.assert_array_equal(np.asarray(vals).reshape(3, 128), values)
        vals2, _ = await store.async_lookup_or_insert(keys, dim=128)
        np.testing.assert_array_equal(np.asarray(vals2), np.asarray(vals))
        await store.async_accumulate_gradients(keys, grads)
        await store.async_optimizer_step(1)
        await store.async_assign_scores(keys, scores)
        after, _ = await store.async_lookup(keys, dim=128)
        mask = await store.async_contains(keys)
        assert np.all(np.asarray(mask) == 1)
        await store.async_erase(keys)
        assert np.all(np.asarray(await store.async_contains(keys)) == 0)
        await store.async_assign(keys, values)
        await store.async_clear()
        assert np.all(np.asarray(await store.async_contains(keys)) == 0)
        return after

    after = asyncio.run(run())
    twin.assign(keys, values)
    twin.lookup_or_insert(keys, 128)
    twin.accumulate_gradients(keys, grads)
    twin.optimizer_step(1)
    np.testing.assert_array_equal(np.asarray(after), np.asarray(twin.lookup(keys, 128)[0]))


def test_async_argument_errors_raise_immediately():
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[8], enable_optimizer=False))

    async def run():
        with pytest.raises(ValueError, match="dim must be > 0"):
            store.async_lookup(np.array([1], np.int64), 0)
        with pytest.raises(RuntimeError, match="async_accumulate_gradients requires optimizer enabled"):
            store.async_accumulate_gradients(np.array([1], np.int64), np.zeros((1, 8), np.float32))
        with pytest.raises(RuntimeError, match="async_optimizer_step requires optimizer enabled"):
            store.async_optimizer_step(1)

    asyncio.run(run())


def test_async_cuda_tensors_and_deferred_error():
    """CUDA inputs run on the caller's stream; an error that the sync call
    defers to the next synchronising call (a device gradient batch that
    fails validation) completes the future with that exception."""
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[4], value_dtype="float16", optimizer_dtype="float32",
                                                 gradient_dtype="float32", key_dtype="int64"),
                              optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    keys = torch.tensor([1, 2], dtype=torch.int64, device="cuda")

    async def run():
        await store.async_lookup_or_insert(keys, 4)
        await store.async_accumulate_gradients(keys, torch.full((2, 4), 1e6, device="cuda"))
        with pytest.raises(OverflowError, match="gradient"):
            await store.async_optimizer_step(1)
        vals, _ = await store.async_lookup(keys, 4)
        return vals

    vals = asyncio.run(run())
    assert torch.equal(vals.cpu().float(), torch.zeros(8))


@pytest.mark.parametrize("accumulation", ["ordered", "atomic"])
def test_clear_discards_keys_and_pending_gradients(accumulation):
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[16, 32], key_dtype="uint64", accumulation=accumulation),
                              optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    keys = np.arange(1, 1001, dtype=np.uint64)
    store.lookup_or_insert(keys, 16)
    store.lookup_or_insert(keys[:10], 32)
    store.accumulate_gradients(keys, np.ones((1000, 16), np.float32))
    assert store.total_size() == 1010
    store.clear()
    assert store.total_size() == 0
    assert np.all(np.asarray(store.contains(keys)) == 0)
    store.optimizer_step(1)  # nothing pending: the cleared window applied nothing
    vals, _ = store.lookup_or_insert(keys, 16)
    assert np.all(np.asarray(vals) == 0.0)
    store.accumulate_gradients(keys, np.ones((1000, 16), np.float32))
    store.optimizer_step(1)
    np.testing.assert_array_equal(np.asarray(store.lookup(keys, 16)[0]), -1.0)
    assert store.total_size() == 1000
