"""The seeded workload generators that build batches on the device, run on
the CPU: determinism, shapes, laws the benches state, and the encode_keys
layout (CPU only)."""

import numpy as np
import torch

from sparse_embedding_b200.workloads import CapacityWorkload, DlrmWorkload, splitmix64_sequence


def test_capacity_device_keys_equal_splitmix64_sequence():
    wl = CapacityWorkload(num_keys=1000)
    got = wl.device_keys(123, 500, torch, device="cpu").view(torch.int64).numpy().view(np.uint64)
    assert np.array_equal(got, splitmix64_sequence(np.arange(123, 623)))


def test_capacity_device_batch_law():
    wl = CapacityWorkload(num_keys=50_000, batch=8192, new_fraction=0.01)
    k1, g1 = wl.device_batch(3, torch, device="cpu")
    k2, g2 = wl.device_batch(3, torch, device="cpu")
    assert torch.equal(k1.view(torch.int64), k2.view(torch.int64)) and torch.equal(g1, g2)
    warmed = set(splitmix64_sequence(np.arange(wl.num_keys)).tolist())
    keys = k1.view(torch.int64).numpy().view(np.uint64).tolist()
    new = [k for k in keys if k not in warmed]
    assert len(new) == round(wl.batch * wl.new_fraction)
    assert g1.shape == (wl.batch, wl.dim) and abs(float(g1.std()) - wl.sigma) < 1e-4


def test_dlrm_device_bags_layout():
    wl = DlrmWorkload(batch=96)
    keys, offsets, bag, pooled = wl.device_bags(1, torch, device="cpu")
    n = keys.numel()
    assert offsets.shape == (wl.batch * wl.tables + 1,) and int(offsets[0]) == 0 and int(offsets[-1]) == n
    counts = offsets[1:] - offsets[:-1]
    assert int(counts.min()) >= 1
    assert torch.equal(bag, torch.repeat_interleave(torch.arange(wl.batch * wl.tables), counts))
    assert pooled.shape == (wl.batch * wl.tables, wl.dim)
    assert 15 < n / (wl.batch * wl.tables) < 25  # max(1, Poisson(20))
    again = wl.device_bags(1, torch, device="cpu")
    assert torch.equal(keys.view(torch.int64), again[0].view(torch.int64))
    other = wl.device_bags(2, torch, device="cpu")
    assert not torch.equal(keys[:100].view(torch.int64), other[0][:100].view(torch.int64))
    # keys of different tables never collide: the table is in bits 40.. of the fmix64 input
    assert torch.unique(keys.view(torch.int64)).numel() <= n


def test_encode_keys_layout_sends_every_table_to_shard_zero_under_fast_range():
    ids = torch.tensor([0, 1, 39_999_999, (1 << 48) - 1, (1 << 60) + 5], dtype=torch.int64)
    for t in (0, 1, 25, 8191, 8192, 65535):
        enc = DlrmWorkload.encode_keys_like(ids, t).numpy().view(np.uint64)
        mask = (1 << 48) - 1
        want = [(t << 48) | (int(i) & mask) for i in ids.tolist()]
        assert [int(x) for x in enc] == want
        # fast_range(key, 8) = (key * 8) >> 64 = key >> 61 = t >> 13
        shards = [(int(x) * 8) >> 64 for x in enc]
        assert shards == [t >> 13] * len(want)
