"""Scores and dynamic learning rates on the GPU (GPU): the reference's known
answers for every policy (tests/test_dynamic_lr.py), LFU/LRU scores equal to
the oracle's after the same lookups, and training with per-row learning
rates against the oracle."""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O
from tests.test_gpu_store import ATOL_FP32, RTOL_FP32, bits

pytestmark = pytest.mark.gpu

DIM = 16

CASES = [
    (se.ConstantLrPolicy(), ("constant", {}), 37, 1.0),
    (se.SqrtDecayLrPolicy(), ("sqrt", {}), 0, 1.0),
    (se.SqrtDecayLrPolicy(), ("sqrt", {}), 4, 0.5),
    (se.LogDecayLrPolicy(), ("log", {}), 2, 0.5),
    (se.InverseDecayLrPolicy(), ("inverse", {}), 0, 1.0),
    (se.InverseDecayLrPolicy(), ("inverse", {}), 4, 0.25),
    (se.CosineFrequencyLrPolicy(min_lr_ratio=0.2, max_score=4), ("cosine", {"lr_min_ratio": 0.2, "lr_max_score": 4}), 2, 0.6),
    (se.CosineFrequencyLrPolicy(min_lr_ratio=0.2, max_score=4), ("cosine", {"lr_min_ratio": 0.2, "lr_max_score": 4}), 5, 0.2),
    (se.CustomLutLrPolicy(lut=[0.25, 0.5, 0.75]), ("lut", {"lr_lut": [0.25, 0.5, 0.75]}), 2, 0.75),
    (se.CustomLutLrPolicy(lut=[0.25, 0.5, 0.75]), ("lut", {"lr_lut": [0.25, 0.5, 0.75]}), 3, 0.75),
]


def make_store(policy, optimizer=se.Sgd, score_policy="manual", lr=1.0):
    return se.EmbeddingStore(se.EmbeddingConfig(dims=[DIM], thread_budget=1, value_dtype="float32"),
                             initializer_config=se.Zeros(), optimizer_config=optimizer(lr=lr, dynamic_lr_policy=policy),
                             score_policy=score_policy)


@pytest.mark.parametrize("policy,orc_policy,score,expected", CASES)
def test_sgd_policy_exact_update(policy, orc_policy, score, expected):
    store = make_store(policy)
    keys = np.array([7], dtype=np.int64)
    store.lookup_or_insert(keys, DIM)
    store.assign_scores(keys, np.array([score], dtype=np.uint64))
    store.accumulate_gradients(keys, np.ones((1, DIM), dtype=np.float32))
    store.optimizer_step(1)
    got = -np.asarray(store.lookup(keys, DIM)[0])
    np.testing.assert_allclose(got, expected, atol=1e-6)
    name, kw = orc_policy
    orc = O.OracleStore([DIM], key_dtype="int64", init="zeros", optimizer="sgd", lr=1.0, score_policy="manual",
                        lr_policy=name, **kw)
    orc.lookup_or_insert(keys, DIM)
    orc.assign_scores(keys, np.array([score], dtype=np.uint64))
    orc.accumulate_gradients(keys, np.ones((1, DIM), dtype=np.float32), DIM)
    orc.optimizer_step(1)
    if name == "log":  # the device log2f and the host's may differ in the last bit
        np.testing.assert_allclose(got, -orc.lookup(keys, DIM), rtol=2e-7)
    else:
        np.testing.assert_array_equal(bits(got), bits(-orc.lookup(keys, DIM)))


def test_adam_applies_exact_dynamic_lr_across_steps():
    store = make_store(se.InverseDecayLrPolicy(), se.Adam)
    keys = np.array([11], dtype=np.int64)
    store.lookup_or_insert(keys, DIM)
    store.assign_scores(keys, np.array([4], dtype=np.uint64))
    for _ in range(2):
        store.accumulate_gradients(keys, np.ones((1, DIM), dtype=np.float32))
        store.optimizer_step(1)
    np.testing.assert_allclose(np.asarray(store.lookup(keys, DIM)[0]), -0.5, atol=2e-5)


@pytest.mark.parametrize("score_policy", ["lfu", "lru"])
def test_runtime_scores_match_the_oracle_and_drive_the_lr(score_policy):
    rng = np.random.default_rng(41)
    gpu = make_store(se.CosineFrequencyLrPolicy(min_lr_ratio=0.1, max_score=100), score_policy=score_policy, lr=0.1)
    orc = O.OracleStore([DIM], key_dtype="int64", init="zeros", optimizer="sgd", lr=0.1, score_policy=score_policy,
                        lr_policy="cosine", lr_min_ratio=0.1, lr_max_score=100)
    pool = np.arange(1, 3001, dtype=np.int64)
    gpu.lookup_or_insert(pool, DIM)
    orc.lookup_or_insert(pool, DIM)
    for i in range(5):
        batch = np.concatenate([rng.choice(pool, size=20_000), rng.integers(10_000, 20_000, size=500)])  # some misses
        if i % 2:
            gpu.lookup(torch.from_numpy(batch).cuda(), DIM)
        else:
            gpu.lookup(batch, DIM)
        orc.lookup(batch, DIM)
    np.testing.assert_array_equal(np.asarray(gpu.read_scores(pool)), orc.read_scores(pool))
    g = np.ones((len(pool), DIM), dtype=np.float32)
    gpu.accumulate_gradients(pool, g)
    orc.accumulate_gradients(pool, g, DIM)
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    got, _ = gpu.lookup(pool, DIM)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(pool, DIM)))


def test_hot_key_gets_a_smaller_update():
    """tests/test_dynamic_lr.py:86-104 on the GPU store."""
    for score_policy in ("lfu", "lru"):
        store = make_store(se.CosineFrequencyLrPolicy(min_lr_ratio=0.1, max_score=100), score_policy=score_policy)
        hot, cold = np.array([1], dtype=np.int64), np.array([2], dtype=np.int64)
        store.lookup_or_insert(hot, DIM)
        store.lookup_or_insert(cold, DIM)
        for _ in range(20):
            store.lookup(hot, DIM)
        g = np.ones((1, DIM), dtype=np.float32)
        store.accumulate_gradients(hot, g)
        store.accumulate_gradients(cold, g)
        store.optimizer_step(1)
        assert np.all(-np.asarray(store.lookup(hot, DIM)[0]) < -np.asarray(store.lookup(cold, DIM)[0]))


def test_adagrad_and_adam_train_with_per_row_rates():
    rng = np.random.default_rng(43)
    for opt, name, kw in ((se.Adagrad, "adagrad", {"initial_accumulator_value": 0.1}), (se.Adam, "adam", {})):
        okw = dict(kw)
        gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[32], key_dtype="int64"),
                                optimizer_config=opt(lr=0.01, dynamic_lr_policy=se.SqrtDecayLrPolicy(), **okw),
                                score_policy="lfu")
        orc = O.OracleStore([32], key_dtype="int64", optimizer=name, lr=0.01, score_policy="lfu", lr_policy="sqrt",
                            initial_accumulator=kw.get("initial_accumulator_value", 0.0))
        pool = rng.integers(-2**63, 2**63 - 1, size=2000, dtype=np.int64)
        gpu.lookup_or_insert(pool, 32)
        orc.lookup_or_insert(pool, 32)
        for _ in range(3):
            batch = rng.choice(pool, size=8000)
            gpu.lookup(batch, 32)
            orc.lookup(batch, 32)
            gr = (rng.standard_normal((len(batch), 32)) * 1e-2).astype(np.float32)
            gpu.accumulate_gradients(batch, gr)
            orc.accumulate_gradients(batch, gr, 32)
            gpu.optimizer_step(1)
            orc.optimizer_step(1)
        got, _ = gpu.lookup(pool, 32)
        np.testing.assert_allclose(got, orc.lookup(pool, 32), rtol=RTOL_FP32, atol=ATOL_FP32)


def test_scores_reset_for_reinserted_keys_and_errors():
    store = make_store(se.SqrtDecayLrPolicy(), score_policy="lfu")
    keys = np.arange(1, 6, dtype=np.int64)
    store.lookup_or_insert(keys, DIM)
    store.lookup(keys, DIM)
    store.lookup(keys, DIM)
    assert np.asarray(store.read_scores(keys)).tolist() == [2] * 5
    store.erase(keys[:2])
    store.lookup_or_insert(keys[:2], DIM)
    assert np.asarray(store.read_scores(keys)).tolist() == [0, 0, 2, 2, 2]
    with pytest.raises(ValueError, match="row counts differ"):
        store.assign_scores(keys, np.zeros(3, dtype=np.uint64))
    plain = se.EmbeddingStore(se.EmbeddingConfig(dims=[DIM]), optimizer_config=se.Sgd())
    with pytest.raises(RuntimeError, match="score-enabled policy"):
        plain.assign_scores(keys, np.zeros(5, dtype=np.uint64))
    with pytest.raises(ValueError, match="requires a score policy"):
        make_store(se.SqrtDecayLrPolicy(), score_policy="none")
    with pytest.raises(ValueError, match="unknown score policy"):
        make_store(se.ConstantLrPolicy(), score_policy="lfx")
