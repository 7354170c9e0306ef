"""Checkpoint interop on the GPU (GPU): export of every present key with its
rows, optimizer state and Adam step, loaded into a fresh store through
assign + assign_opt_state, gives a store identical bit for bit (and it keeps
training identically); exported contents equal the oracle's."""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from sparse_embedding_b200 import checkpoint as ck
from tests.test_gpu_store import bits, pair

pytestmark = pytest.mark.gpu


def trained(value_dtype="float32", optimizer_dtype="", opt="adam", dims=(16, 32)):
    rng = np.random.default_rng(31)
    gpu, orc = pair(list(dims), key_dtype="int64", value_dtype=value_dtype, optimizer_dtype=optimizer_dtype,
                    opt=opt, lr=1e-2)
    pool = rng.integers(-2**63, 2**63 - 1, size=6000, dtype=np.int64)
    inserted = {d: set() for d in dims}
    for d in dims:
        for step in range(3):
            keys = rng.choice(pool, size=4000)
            inserted[d].update(keys.tolist())
            gpu.lookup_or_insert(keys, d)
            orc.lookup_or_insert(keys, d)
            g = (rng.standard_normal((len(keys), d)) * 1e-2).astype(np.float32)
            if gpu.gradient_dtype() != "float32":
                g = torch.from_numpy(g).to(torch.bfloat16 if gpu.gradient_dtype() == "bfloat16" else torch.float16)
            gpu.accumulate_gradients(keys, g)
            gpu.optimizer_step(1)
    gone = np.ascontiguousarray(pool[::7])
    gpu.erase(gone)
    orc.erase(gone)
    present = {d: np.array(sorted(inserted[d] - set(gone.tolist())), dtype=np.int64) for d in dims}
    return gpu, orc, present


def collect(store, **kw):
    out = {}
    for batch in ck.export_batches(store, batch_size=1500, **kw):
        d = batch[0]
        out.setdefault(d, []).append(batch[1:])
    merged = {}
    for d, parts in out.items():
        merged[d] = [np.concatenate([np.asarray(bits(p[i])) for p in parts]) for i in range(len(parts[0]))]
    return merged


@pytest.mark.parametrize("value_dtype,optimizer_dtype", [("float32", ""), ("bfloat16", "float32"), ("float16", "float16")])
def test_export_then_import_reproduces_the_store(value_dtype, optimizer_dtype):
    gpu, orc, present = trained(value_dtype, optimizer_dtype)
    exp = collect(gpu, include_optimizer_state=True, include_steps=True)
    assert sum(len(v[0]) for v in exp.values()) == gpu.total_size() == orc.size()
    fresh, _ = pair([16, 32], key_dtype="int64", value_dtype=value_dtype, optimizer_dtype=optimizer_dtype,
                    opt="adam", lr=1e-2)
    for batch in ck.export_batches(gpu, batch_size=1500, include_optimizer_state=True, include_steps=True):
        d, keys, vals, states, steps = batch
        fresh.assign(keys, vals)
        ck.assign_opt_state(fresh, keys, states, d, steps)
    for d in (16, 32):
        keys, vals, states, steps = exp[d]
        assert len(np.unique(keys)) == len(keys)
        np.testing.assert_array_equal(np.sort(keys), present[d])
        got, _ = fresh.lookup(keys, d)
        np.testing.assert_array_equal(bits(got).reshape(len(keys), d), vals.reshape(len(keys), d))
        got, _ = gpu.lookup(keys, d)
        np.testing.assert_array_equal(bits(got).reshape(len(keys), d), vals.reshape(len(keys), d))
        for i in range(0, len(keys), 997):
            f1, p1, s1, t1 = gpu.read_state(int(keys[i]), d)
            f2, p2, s2, t2 = fresh.read_state(int(keys[i]), d)
            assert f1 and f2 and t1 == t2 == steps[i]
            np.testing.assert_array_equal(bits(s1), bits(s2))
            np.testing.assert_array_equal(bits(s1), states[i])
    # both keep training identically
    rng = np.random.default_rng(5)
    keys = np.ascontiguousarray(exp[16][0][:3000])
    g = (rng.standard_normal((len(keys), 16)) * 1e-2).astype(np.float32)
    if gpu.gradient_dtype() != "float32":
        g = torch.from_numpy(g).to(torch.bfloat16 if gpu.gradient_dtype() == "bfloat16" else torch.float16)
    for s in (gpu, fresh):
        s.accumulate_gradients(keys, g)
        s.optimizer_step(1)
    np.testing.assert_array_equal(bits(gpu.lookup(keys, 16)[0]), bits(fresh.lookup(keys, 16)[0]))


def test_exported_rows_equal_the_oracle_and_the_visitor_form():
    gpu, orc = pair([8], key_dtype="uint64", opt="adagrad", lr=0.01, initial_accumulator_value=0.1)
    keys = np.random.default_rng(2).integers(0, 2**64 - 1, size=20_000, dtype=np.uint64)
    keys = np.concatenate([keys, np.array([2**64 - 1, 0], dtype=np.uint64)])  # the all-ones key too
    gpu.lookup_or_insert(keys, 8)
    orc.lookup_or_insert(keys, 8)
    seen = []
    ck.export_batches_dlpack(gpu, lambda d, k, v, s: seen.append((d, k, v, s)), batch_size=4096,
                             include_optimizer_state=True)
    assert all(len(b[1]) <= 4096 for b in seen) and sum(len(b[1]) for b in seen) == orc.size()
    k = np.concatenate([b[1] for b in seen])
    v = np.concatenate([b[2] for b in seen])
    s = np.concatenate([b[3] for b in seen])
    np.testing.assert_array_equal(np.sort(k), np.unique(keys))
    np.testing.assert_array_equal(v.reshape(-1).view(np.uint32), orc.lookup(k, 8).view(np.uint32))
    assert s.shape == (len(k), 8) and (s == np.float32(0.1)).all()


def test_assign_opt_state_errors_leave_the_store_unchanged():
    gpu, _ = pair([8], key_dtype="int64", opt="adam", lr=1e-3)
    keys = np.arange(10, dtype=np.int64)
    gpu.lookup_or_insert(keys, 8)
    states = np.ones((11, 16), dtype=np.float32)
    with pytest.raises(ValueError, match="absent from dimension table"):
        ck.assign_opt_state(gpu, np.arange(11, dtype=np.int64), states, 8)
    assert (gpu.read_state(3, 8)[2] == 0).all()
    with pytest.raises(ValueError, match="payload size does not match"):
        ck.assign_opt_state(gpu, keys, np.ones((10, 8), dtype=np.float32), 8)
    with pytest.raises(ValueError, match="no physical table"):
        ck.assign_opt_state(gpu, keys, np.ones((10, 16), dtype=np.float32), 16)
    ck.assign_opt_state(gpu, keys, states[:10], 8, np.full(10, 7, dtype=np.uint32))
    f, _, s, t = gpu.read_state(3, 8)
    assert f and t == 7 and (s == 1).all()
    sgd, _ = pair([8], key_dtype="int64", opt="sgd")
    sgd.lookup_or_insert(keys, 8)
    with pytest.raises(ValueError, match="payload size does not match"):
        ck.assign_opt_state(sgd, keys, np.ones((10, 8), dtype=np.float32), 8)


@pytest.mark.parametrize("value_dtype,opt", [("float32", "adam"), ("bfloat16", "adagrad"), ("float32", "sgd")])
def test_page_images_round_trip(value_dtype, opt):
    """export_page_images -> import_page_images into an empty store of the
    same configuration reproduces every key's row, optimizer state and Adam
    step (page dicts with the reference's fields), and the copy trains on
    identically; the reference's import errors are kept."""
    gpu, _, present = trained(value_dtype=value_dtype, opt=opt)
    pages = gpu.export_page_images()
    assert pages and {"embedding_dim", "physical_page_id", "page_slot_stride_bytes", "slot_ordinals", "keys",
                      "seq_counts", "scores", "steps", "values", "optimizer_states"} <= set(pages[0])
    per_page = gpu.entries_per_page
    assert all(len(p["keys"]) <= per_page for p in pages)
    assert sum(len(p["keys"]) for p in pages) == gpu.total_size()
    fresh, _ = pair([16, 32], key_dtype="int64", value_dtype=value_dtype, opt=opt, lr=1e-2)
    fresh.import_page_images(pages)
    assert fresh.total_size() == gpu.total_size()
    for d, keys in present.items():
        np.testing.assert_array_equal(bits(fresh.lookup(keys, d)[0]), bits(gpu.lookup(keys, d)[0]))
        for k in keys[:20]:
            a, b = gpu.read_state(int(k), d), fresh.read_state(int(k), d)
            assert a[0] and b[0] and a[3] == b[3]
            np.testing.assert_array_equal(a[2], b[2])
    rng = np.random.default_rng(5)
    keys = rng.choice(present[16], size=3000)
    g = (rng.standard_normal((len(keys), 16)) * 1e-2).astype(np.float32)
    if value_dtype == "bfloat16":
        g = torch.from_numpy(g).to(torch.bfloat16)
    for s in (gpu, fresh):
        s.accumulate_gradients(keys, g)
        s.optimizer_step(1)
    np.testing.assert_array_equal(bits(fresh.lookup(present[16], 16)[0]), bits(gpu.lookup(present[16], 16)[0]))
    with pytest.raises(RuntimeError, match="requires empty slots"):
        fresh.import_page_images(pages)
    other, _ = pair([8], key_dtype="int64", value_dtype=value_dtype, opt=opt, lr=1e-2)
    with pytest.raises(ValueError, match="no physical table"):
        other.import_page_images(pages)
    empty, _ = pair([16, 32], key_dtype="int64", value_dtype=value_dtype, opt=opt, lr=1e-2)
    with pytest.raises(ValueError, match="duplicate page ids"):
        empty.import_page_images([pages[0], pages[0]])
