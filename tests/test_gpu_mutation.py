"""Mutation API on the GPU against the CPU oracle (GPU): assign, contains,
erase and erase_dimension, through the C ABI.

Cases follow the reference's tests: assign then lookup reads the values back
exactly (tests/test_embedding_table.py:89-106, test_mixed_precision.py:112-140),
assign shape errors (test_ops.py:348-370), erase then insert keeps the size
(test_embedding_table.py:207-222), erase/reinsert/contains
(mutation_contract_test.cpp:23-95). Gathered and inserted rows are
bit-exact; rows updated by the optimizer within the fp32 tolerance of the
store tests.
"""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from tests.test_gpu_store import ATOL_FP32, RTOL_FP32, bits, pair

pytestmark = pytest.mark.gpu


def rand_values(n, dim, dtype, rng):
    """(input for the GPU store, raw array for the oracle) of n rows."""
    v = rng.uniform(-1, 1, (n, dim)).astype(np.float32)
    if dtype == "float32":
        return v, v
    if dtype == "float16":
        h = v.astype(np.float16)
        return h, h.view(np.uint16)
    t = torch.from_numpy(v).to(torch.bfloat16)
    return t, bits(t)


@pytest.mark.parametrize("value_dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("key_dtype", ["int64", "uint64", "int32", "uint32"])
def test_assign_then_lookup_is_exact(value_dtype, key_dtype):
    rng = np.random.default_rng(1)
    dim = 24
    gpu, orc = pair([dim], key_dtype=key_dtype, value_dtype=value_dtype, opt="adam")
    keys = rng.choice(np.arange(1, 10_000), size=500, replace=False).astype(key_dtype)
    warm = keys[:200]
    gpu.lookup_or_insert(warm, dim)
    orc.lookup_or_insert(warm, dim)
    vg, vr = rand_values(len(keys), dim, value_dtype, rng)
    gpu.assign(keys, vg)
    orc.assign(keys, vr, dim)
    assert gpu.total_size() == orc.size() == len(keys)
    got, _ = gpu.lookup(keys, dim)
    np.testing.assert_array_equal(bits(got).reshape(-1), bits(vr).reshape(-1))
    np.testing.assert_array_equal(bits(got).reshape(-1), bits(orc.lookup(keys, dim)))


def test_assign_keeps_optimizer_state_and_trains_like_the_oracle():
    rng = np.random.default_rng(2)
    dim = 32
    gpu, orc = pair([dim], opt="adam", lr=1e-2)
    keys = np.arange(100, 400, dtype=np.int64)
    gpu.lookup_or_insert(keys, dim)
    orc.lookup_or_insert(keys, dim)
    g = (rng.standard_normal((len(keys), dim)) * 1e-2).astype(np.float32)
    gpu.accumulate_gradients(keys, g)
    orc.accumulate_gradients(keys, g, dim)
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    # half present, half new
    akeys = np.arange(250, 550, dtype=np.int64)
    vals = rng.uniform(-0.1, 0.1, (len(akeys), dim)).astype(np.float32)
    gpu.assign(akeys, vals)
    orc.assign(akeys, vals, dim)
    for k in (250, 399, 400, 549):
        f1, p1, s1, t1 = gpu.read_state(k, dim)
        f2, p2, s2, t2 = orc.read_row(k, dim, nstate=2)
        assert f1 and f2 and t1 == t2 == (1 if k < 400 else 0)
        np.testing.assert_array_equal(bits(p1), bits(p2))
        np.testing.assert_array_equal(bits(s1), bits(s2.view(np.float32)))
    allk = np.arange(100, 550, dtype=np.int64)
    g2 = (rng.standard_normal((len(allk), dim)) * 1e-2).astype(np.float32)
    gpu.accumulate_gradients(allk, g2)
    orc.accumulate_gradients(allk, g2, dim)
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    got, _ = gpu.lookup(allk, dim)
    np.testing.assert_allclose(np.asarray(got), orc.lookup(allk, dim).reshape(np.asarray(got).shape),
                               rtol=RTOL_FP32, atol=ATOL_FP32)


def test_contains_erase_and_reinsert_match_the_oracle():
    rng = np.random.default_rng(3)
    dim = 16
    gpu, orc = pair([dim], key_dtype="int64", opt="adagrad", lr=0.01, eps=1e-8, initial_accumulator_value=0.1)
    pool = rng.integers(-2**63, 2**63 - 1, size=5000, dtype=np.int64)
    pool = np.concatenate([pool, np.array([0, -1, -2**63, 2**63 - 1], dtype=np.int64)])  # -1 = all-ones key
    gpu.lookup_or_insert(pool, dim)
    orc.lookup_or_insert(pool, dim)
    probe = np.concatenate([pool[::7], rng.integers(-2**63, 2**63 - 1, size=300, dtype=np.int64)])
    np.testing.assert_array_equal(np.asarray(gpu.contains(probe)), orc.contains(probe))
    # erase a third (with repeats and absent keys), on host and then on device inputs
    gone = np.concatenate([pool[::3], pool[::9], np.array([-1, 12345], dtype=np.int64)])
    gpu.erase(gone[: len(gone) // 2])
    orc.erase(gone[: len(gone) // 2])
    gpu.erase(torch.from_numpy(gone[len(gone) // 2:]).cuda())
    orc.erase(gone[len(gone) // 2:])
    assert gpu.total_size() == orc.size()
    np.testing.assert_array_equal(np.asarray(gpu.contains(pool)), orc.contains(pool))
    dev = gpu.contains(torch.from_numpy(pool).cuda())
    assert dev.dtype == torch.uint8 and dev.is_cuda
    np.testing.assert_array_equal(dev.cpu().numpy(), orc.contains(pool))
    # erased keys read as zeros; reinserted keys get their initializer row again
    got, _ = gpu.lookup(pool, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(pool, dim)))
    back = np.ascontiguousarray(gone[::2])
    got, _ = gpu.lookup_or_insert(back, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup_or_insert(back, dim)))
    # new keys take the erased keys' rows
    fresh = rng.integers(-2**63, 2**63 - 1, size=3000, dtype=np.int64)
    got, _ = gpu.lookup_or_insert(fresh, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup_or_insert(fresh, dim)))
    assert gpu.total_size() == orc.size()
    everything = np.concatenate([pool, fresh])
    got, _ = gpu.lookup(everything, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(everything, dim)))
    # the reinserted keys start their optimizer state again
    for k in back[:8]:
        f1, _, s1, _ = gpu.read_state(int(k), dim)
        f2, _, s2, _ = orc.read_row(int(k), dim, nstate=1)
        assert f1 and f2
        np.testing.assert_array_equal(bits(s1), bits(s2.view(np.float32)))


def test_erase_then_insert_keeps_total_size():
    """tests/test_embedding_table.py:207-222 on the GPU store."""
    gpu, orc = pair([8], init="zeros", opt="sgd")
    keys = np.arange(8193, dtype=np.int64)
    gpu.lookup_or_insert(keys, 8)
    assert gpu.total_size() == len(keys)
    gpu.erase(np.array([1], dtype=np.int64))
    assert gpu.total_size() == len(keys) - 1
    gpu.lookup_or_insert(np.array([8193], dtype=np.int64), 8)
    assert gpu.total_size() == len(keys)


def test_erase_many_then_grow_past_the_directory():
    """Tombstones count toward the directory's load until a rehash drops them."""
    rng = np.random.default_rng(4)
    dim = 8
    gpu, orc = pair([dim], key_dtype="uint64", opt="sgd", capacity=4096)
    live = np.array([], dtype=np.uint64)
    for r in range(6):
        add = rng.integers(0, 2**64 - 1, size=3000, dtype=np.uint64)
        gpu.lookup_or_insert(add, dim)
        orc.lookup_or_insert(add, dim)
        live = np.concatenate([live, add])
        drop = live[rng.random(len(live)) < 0.5]
        gpu.erase(drop)
        orc.erase(drop)
        assert gpu.total_size() == orc.size()
    got, _ = gpu.lookup(live, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(live, dim)))
    np.testing.assert_array_equal(np.asarray(gpu.contains(live)), orc.contains(live))


def test_erase_with_pending_gradients():
    """Gradients of a key erased before the step are dropped (counted); a key
    erased and inserted again before the step gets them on its new row."""
    rng = np.random.default_rng(5)
    dim = 16
    gpu, orc = pair([dim], opt="adam", lr=1e-2)
    keys = np.arange(1, 2001, dtype=np.int64)
    gpu.lookup_or_insert(keys, dim)
    orc.lookup_or_insert(keys, dim)
    batch = rng.choice(keys, size=6000)  # repeats: several rows per key
    g = (rng.standard_normal((len(batch), dim)) * 1e-2).astype(np.float32)
    gpu.accumulate_gradients(batch, g)
    orc.accumulate_gradients(batch, g, dim)
    gone = np.ascontiguousarray(keys[::4])
    gpu.erase(gone)
    orc.erase(gone)
    back = np.ascontiguousarray(gone[::3])
    got, _ = gpu.lookup_or_insert(back, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup_or_insert(back, dim)))
    # a device batch after the erase joins the same window
    b2 = rng.choice(keys, size=1000)
    g2 = (rng.standard_normal((len(b2), dim)) * 1e-2).astype(np.float32)
    gpu.accumulate_gradients(torch.from_numpy(b2).cuda(), torch.from_numpy(g2).cuda())
    orc.accumulate_gradients(b2, g2, dim)
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    assert gpu.dropped_gradients() == orc.dropped() > 0
    got, _ = gpu.lookup(keys, dim)
    np.testing.assert_allclose(np.asarray(got), orc.lookup(keys, dim).reshape(np.asarray(got).shape),
                               rtol=RTOL_FP32, atol=ATOL_FP32)
    for k in back[:6]:
        f1, _, _, t1 = gpu.read_state(int(k), dim)
        f2, _, _, t2 = orc.read_row(int(k), dim, nstate=2)
        assert f1 and f2 and t1 == t2


def test_bulk_inserts_into_recycled_rows():
    """Whole batches of new keys after large erases: rows come off the free
    stack a warp at a time, partly from it and partly from the arena's end."""
    rng = np.random.default_rng(6)
    dim = 32
    gpu, orc = pair([dim], key_dtype="uint64", opt="adam", lr=1e-2, capacity=1 << 16)
    base = rng.integers(0, 2**64 - 1, size=40_000, dtype=np.uint64)
    gpu.lookup_or_insert(base, dim)
    orc.lookup_or_insert(base, dim)
    for r in range(3):
        gone = np.ascontiguousarray(base[r * 10_000:(r + 1) * 10_000 - 37 * r])
        gpu.erase(gone)
        orc.erase(gone)
        fresh = rng.integers(0, 2**64 - 1, size=10_000 + 5_000 * r, dtype=np.uint64)
        got, _ = gpu.lookup_or_insert(torch.from_numpy(fresh.view(np.int64)).cuda().view(torch.uint64), dim)
        np.testing.assert_array_equal(bits(got), bits(orc.lookup_or_insert(fresh, dim)))
        vals = rng.uniform(-1, 1, (4_000, dim)).astype(np.float32)
        akeys = np.unique(rng.integers(0, 2**64 - 1, size=4_000, dtype=np.uint64))
        gpu.assign(akeys, vals[: len(akeys)])
        orc.assign(akeys, vals[: len(akeys)], dim)
        assert gpu.total_size() == orc.size()
        base = np.concatenate([base, fresh, akeys])
    got, _ = gpu.lookup(base, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(base, dim)))


def test_erase_dimension_touches_one_table():
    gpu, orc = pair([8, 32], opt="sgd")
    keys = np.arange(1000, dtype=np.int64)
    for d in (8, 32):
        gpu.lookup_or_insert(keys, d)
        orc.lookup_or_insert(keys, d)
    gpu.erase_dimension(keys[:500], 32)
    orc.erase(keys[:500], dim=32)
    assert gpu.size(32) == orc.size(32) == 500 and gpu.size(8) == orc.size(8) == 1000
    np.testing.assert_array_equal(np.asarray(gpu.contains(keys)), orc.contains(keys))
    assert np.asarray(gpu.contains(keys)).all()  # still held by the dim-8 table
    for d in (8, 32):
        got, _ = gpu.lookup(keys, d)
        np.testing.assert_array_equal(bits(got), bits(orc.lookup(keys, d)))
    with pytest.raises(ValueError, match="erase dimension must be non-negative"):
        gpu.erase_dimension(keys, -1)
    with pytest.raises(ValueError, match="erase dimension is not configured"):
        gpu.erase_dimension(keys, 16)


def test_assign_argument_errors():
    """test_ops.py:348-370 and validate_unique_mutation_batch."""
    gpu, _ = pair([128], init="zeros", opt="adam", lr=0.01)
    keys = np.array([1, 2, 3], dtype=np.int64)
    with pytest.raises(ValueError, match="must match keys length"):
        gpu.assign(keys, np.random.rand(1, 128).astype(np.float32))
    with pytest.raises(ValueError, match="multiple of keys length"):
        gpu.assign(keys, np.zeros(10, dtype=np.float32))
    with pytest.raises(ValueError, match="1D or 2D"):
        gpu.assign(keys, np.zeros((3, 2, 64), dtype=np.float32))
    with pytest.raises(ValueError, match="duplicate dimension and key"):
        gpu.assign(np.array([5, 6, 5], dtype=np.int64), np.zeros((3, 128), dtype=np.float32))
    with pytest.raises(ValueError, match="duplicate dimension and key"):
        gpu.assign(torch.tensor([7, 7], dtype=torch.int64, device="cuda"),
                   torch.zeros((2, 128), device="cuda"))
    with pytest.raises(ValueError, match="duplicate dimension and key"):
        gpu.assign(np.array([-1, 3, -1], dtype=np.int64), np.zeros((3, 128), dtype=np.float32))
    with pytest.raises(RuntimeError, match="invalid dim access"):
        gpu.assign(keys, np.zeros((3, 64), dtype=np.float32))
    assert gpu.total_size() == 0
    # device inputs
    v = torch.rand((3, 128), device="cuda")
    gpu.assign(torch.from_numpy(keys).cuda(), v)
    got, _ = gpu.lookup(keys, 128)
    np.testing.assert_array_equal(bits(got).reshape(3, 128), bits(v))


def test_assign_and_erase_through_the_row_length_entry_points():
    """The facade forms with row_lengths (se_assign) against the dim form."""
    import ctypes as C

    from sparse_embedding_b200 import _native as N

    gpu, _ = pair([4], init="zeros", opt="sgd")
    lib = N.lib()
    keys = np.array([11, 12], dtype=np.int64)
    vals = np.arange(8, dtype=np.float32)
    lens = np.array([4, 4], dtype=np.int64)
    N.check(lib.se_assign(gpu._h, keys.ctypes.data, 2, vals.ctypes.data, 8,
                          lens.ctypes.data_as(C.POINTER(C.c_int64)), 2, None))
    got, _ = gpu.lookup(keys, 4)
    np.testing.assert_array_equal(np.asarray(got).reshape(-1), vals)
    out = np.zeros(3, dtype=np.uint8)
    probe = np.array([11, 12, 13], dtype=np.int64)
    N.check(lib.se_contains(gpu._h, probe.ctypes.data, 3, out.ctypes.data, None))
    assert out.tolist() == [1, 1, 0]
    N.check(lib.se_erase(gpu._h, keys.ctypes.data, 1, None))
    N.check(lib.se_contains(gpu._h, probe.ctypes.data, 3, out.ctypes.data, None))
    assert out.tolist() == [0, 1, 0]
    assert np.asarray(gpu.lookup(keys[:1], 4)[0]).tolist() == [0.0] * 4
