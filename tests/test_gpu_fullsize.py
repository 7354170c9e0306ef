"""The bench's train-step workload at full size (GPU): a 10M-key dim-64 fp32
Adagrad table, 65,536-key Zipf(1.05) + 5 % new batches. A key's row depends
only on its initialisation (a function of the key) and its own gradients, so
the full-size store is checked exactly against an oracle holding just the
keys that are looked at: a sample of the warmed table, and every key of the
trained batches."""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O
from sparse_embedding_b200.workloads import TrainWorkload
from tests.test_gpu_store import ATOL_FP32, RTOL_FP32, bits

pytestmark = pytest.mark.gpu


def test_full_size_train_steps_against_the_oracle():
    wl = TrainWorkload()  # 10M warmed keys, 65,536-key batches
    dim = wl.dim
    store = se.EmbeddingStore(
        se.EmbeddingConfig(dims=[dim], key_dtype="int64", initial_capacity=wl.num_keys + 1_000_000),
        optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))
    warm = wl.warm_keys()
    for i in range(0, len(warm), 1 << 20):
        store.lookup_or_insert(torch.from_numpy(warm[i:i + (1 << 20)]).cuda(), dim)
    assert store.total_size() == wl.num_keys
    rng = np.random.default_rng(99)
    sample = warm[rng.choice(len(warm), size=100_000, replace=False)]
    orc = O.OracleStore([dim], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8, initial_accumulator=0.1)
    got, _ = store.lookup(torch.from_numpy(sample).cuda(), dim)
    np.testing.assert_array_equal(bits(got).reshape(-1), bits(orc.lookup_or_insert(sample, dim)))
    before = bits(got).reshape(len(sample), dim).copy()
    # three train steps; the oracle sees only the batches' keys (and the sample)
    keys, grads = wl.make_batches(3, start_step=777)
    for s in range(3):
        k = torch.from_numpy(keys[s]).cuda()
        store.lookup_or_insert(k, dim)
        store.accumulate_gradients(k, torch.from_numpy(grads[s]).cuda())
        store.optimizer_step(1)
        orc.lookup_or_insert(keys[s], dim)
        orc.accumulate_gradients(keys[s], grads[s], dim)
        orc.optimizer_step(1)
    touched = np.unique(keys)
    got, _ = store.lookup(torch.from_numpy(touched).cuda(), dim)
    np.testing.assert_allclose(got.cpu().numpy().reshape(-1, dim), orc.lookup(touched, dim).reshape(-1, dim),
                               rtol=RTOL_FP32, atol=ATOL_FP32)
    # keys no batch touched are unchanged, bit for bit
    untouched = ~np.isin(sample, touched)
    after = bits(store.lookup(torch.from_numpy(sample).cuda(), dim)[0]).reshape(len(sample), dim)
    np.testing.assert_array_equal(after[untouched], before[untouched])
    # the table grew by exactly the batches' new keys
    new_keys = np.setdiff1d(touched, warm)
    assert store.total_size() == wl.num_keys + len(new_keys)
    assert store.dropped_gradients() == 0
