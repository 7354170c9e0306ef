"""The benchmark configurations' workload shapes at sizes the oracle finishes
in seconds, through the public API, against the CPU oracle (GPU).

forward lookup (dim 32, Zipf 1.1 over u64 keys), DLRM-style multi-table
(pre-mixed keys of several tables, dim 128, sum-pooled bags, Adam), capacity
run (u64 keys, Adam, 1% new keys, modulo ownership), weight-only inference
(int32 keys, dim 256 bf16, no optimizer, uniform batches, hash ownership).
Gathers and inserted rows are bit-exact; updated fp32 parameters and state
within 1e-5 relative (hot keys are reduced in parallel runs).
"""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O
from sparse_embedding_b200.workloads import (CapacityWorkload, DlrmWorkload, ForwardWorkload, InferenceWorkload)
from tests.test_gpu_store import ATOL_FP32, RTOL_FP32, bits, pair

pytestmark = pytest.mark.gpu


def test_forward_lookup_workload_bit_exact():
    wl = ForwardWorkload(num_keys=50_000)
    gpu, orc = pair([32], key_dtype="uint64", opt="none")
    warm = wl.warm_keys()
    gpu.lookup_or_insert(warm, 32)
    orc.lookup_or_insert(warm, 32)
    for b in wl.batches(8):
        got, _ = gpu.lookup(b, 32)
        np.testing.assert_array_equal(bits(got), bits(orc.lookup(b, 32)))
    # device-resident batches on the CUDA path
    b = torch.from_numpy(wl.batches(1)[0]).cuda()
    got, _ = gpu.lookup(b, 32)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(b.cpu().numpy(), 32)))


def test_dlrm_multi_table_adam():
    wl = DlrmWorkload(tables=4, min_rows=200, max_rows=20_000, batch=64)
    gpu, orc = pair([128], key_dtype="uint64", opt="adam", lr=1e-3)
    seen = []
    for step in range(3):
        keys, bag, pooled = wl.make_batch(step)
        seen.append(keys)
        rows, _ = gpu.lookup_or_insert(torch.from_numpy(keys).cuda(), 128)
        ref = orc.lookup_or_insert(keys, 128).reshape(-1, 128)
        got = rows.view(-1, 128).cpu().numpy()
        if step == 0:
            np.testing.assert_array_equal(bits(got), bits(ref))
        else:
            np.testing.assert_allclose(got, ref, rtol=RTOL_FP32, atol=ATOL_FP32)
        # harness: sum-pool per (sample, table); pooled gradient back to every id of the bag
        b = torch.from_numpy(bag).cuda()
        pooled_rows = torch.zeros((wl.batch * wl.tables, 128), device="cuda").index_add_(0, b, rows.view(-1, 128))
        assert torch.isfinite(pooled_rows).all()
        grads = pooled[bag]
        gpu.accumulate_gradients(torch.from_numpy(keys).cuda(), torch.from_numpy(grads).cuda())
        orc.accumulate_gradients(keys, grads, 128)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    probe = np.unique(np.concatenate(seen))
    got, _ = gpu.lookup(probe, 128)
    np.testing.assert_allclose(np.asarray(got).reshape(-1, 128), orc.lookup(probe, 128).reshape(-1, 128),
                               rtol=RTOL_FP32, atol=ATOL_FP32)
    for k in probe[:64]:
        found_g, p, s, step = gpu.read_state(int(k), 128)
        found, rp, rs, rstep = orc.read_row(int(k), 128, nstate=2)
        assert found_g and found and step == rstep
        np.testing.assert_allclose(np.asarray(s).ravel(), rs.view(np.float32), rtol=RTOL_FP32, atol=1e-9)


def test_capacity_run_shape_modulo_owner():
    """Rank 1 of 4 under the modulo partitioner: warms only the keys it owns,
    then trains on its share of 16,384-key batches (Zipf 1.05 + 1% new)."""
    wl = CapacityWorkload(num_keys=400_000, batch=16_384)
    part = se.ModuloPartitioner(num_shards=4)
    warm = wl.warm_keys()
    mine = warm[np.asarray(part.partition(warm)) == 1]
    gpu, orc = pair([64], key_dtype="uint64", opt="adam", lr=1e-3, capacity=len(mine) + 10_000)
    gpu.lookup_or_insert(mine, 64)
    orc.lookup_or_insert(mine, 64)
    keys, grads = wl.make_batches(3)
    for s in range(3):
        own = np.asarray(part.partition(keys[s])) == 1
        k, g = keys[s][own], grads[s][own]
        got, _ = gpu.lookup_or_insert(k, 64)
        ref = orc.lookup_or_insert(k, 64)
        np.testing.assert_allclose(np.asarray(got), ref.reshape(np.asarray(got).shape), rtol=RTOL_FP32, atol=ATOL_FP32)
        gpu.accumulate_gradients(k, g)
        orc.accumulate_gradients(k, g, 64)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    assert gpu.total_size() == orc.size()
    sample = np.random.default_rng(3).choice(mine, size=4096, replace=False)
    got, _ = gpu.lookup(sample, 64)
    np.testing.assert_allclose(np.asarray(got), orc.lookup(sample, 64).reshape(np.asarray(got).shape),
                               rtol=RTOL_FP32, atol=ATOL_FP32)


def test_weight_only_inference_bf16_int32():
    wl = InferenceWorkload(num_keys=100_000, batch=32_768)
    gpu, orc = pair([256], key_dtype="int32", value_dtype="bfloat16", opt="none")
    warm = torch.from_numpy(wl.warm_keys()).cuda()
    gpu.lookup_or_insert(warm, 256)
    orc.lookup_or_insert(wl.warm_keys(), 256)
    part = se.HashPartitioner(num_shards=8)
    for b in wl.batches(3):
        got, _ = gpu.lookup(torch.from_numpy(b).cuda(), 256)
        np.testing.assert_array_equal(bits(got), orc.lookup(b, 256))
        # the hash owner of every key matches the oracle's partitioner
        np.testing.assert_array_equal(np.asarray(part.partition(b)), O.partition("hash", 8, b))
