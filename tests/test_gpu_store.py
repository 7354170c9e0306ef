"""Store hot path on the GPU against the CPU oracle, through the C ABI (GPU).

Forward gathers and inserted rows must be bit-identical to the oracle.
Optimizer updates are bit-identical when every key's gradients are reduced
serially (segments up to 64 rows); hot keys reduced in parallel runs must be
within 1e-5 relative (fp32) of the oracle's serial sum.
"""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O
from sparse_embedding_b200.workloads import TrainWorkload, splitmix64_sequence

pytestmark = pytest.mark.gpu

RTOL_FP32 = 1e-5
# Values live in [-0.05, 0.05] (the default initializer) and move by ~1e-3 per
# step, so elements that cross zero are compared at 1e-5 of that scale.
ATOL_FP32 = RTOL_FP32 * 0.05


def bits(x):
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu()
        if x.dtype in (torch.bfloat16, torch.float16):
            return x.view(torch.int16).numpy().view(np.uint16)
        x = x.numpy()
    x = np.asarray(x)
    if x.dtype == np.float32:
        return x.view(np.uint32)
    if x.dtype == np.float16:
        return x.view(np.uint16)
    return x


def as_float(raw, dtype):
    raw = np.asarray(raw)
    if dtype == "float32":
        return raw.astype(np.float32)
    if dtype == "float16":
        return raw.view(np.float16).astype(np.float32)
    return (raw.astype(np.uint32) << 16).view(np.float32)


def make_grads(shape, dtype, rng, scale=1e-2):
    """(input for the GPU store, raw array for the oracle)."""
    g = (rng.standard_normal(shape) * scale).astype(np.float32)
    if dtype == "float32":
        return g, g
    if dtype == "float16":
        h = g.astype(np.float16)
        return h, h.view(np.uint16)
    t = torch.from_numpy(g).to(torch.bfloat16)
    return t, bits(t)


def pair(dims, key_dtype="int64", value_dtype="float32", optimizer_dtype="", gradient_dtype="",
         gradient_scale=1.0, init="uniform", opt="adam", capacity=0, **okw):
    cfg = se.EmbeddingConfig(dims=dims, thread_budget=1, key_dtype=key_dtype, value_dtype=value_dtype,
                             optimizer_dtype=optimizer_dtype, gradient_dtype=gradient_dtype,
                             gradient_scale=gradient_scale, enable_optimizer=opt != "none",
                             initial_capacity=capacity)
    initc = se.Uniform() if init == "uniform" else se.Zeros()
    optc = {"adam": se.Adam, "sgd": se.Sgd, "adagrad": se.Adagrad}.get(opt)
    gpu = se.EmbeddingStore(cfg, initializer_config=initc, optimizer_config=optc(**okw) if optc else None)
    ref_kw = dict(okw)
    if opt == "adagrad":
        ref_kw["initial_accumulator"] = ref_kw.pop("initial_accumulator_value", 0.1)
        ref_kw.setdefault("lr", 1e-2)
    if opt == "sgd":
        ref_kw.setdefault("lr", 1e-2)
    orc = O.OracleStore(dims, key_dtype=key_dtype, value_dtype=value_dtype, optimizer_dtype=optimizer_dtype,
                        gradient_dtype=gradient_dtype, gradient_scale=gradient_scale, enable_optimizer=opt != "none",
                        init=init, optimizer=opt, **ref_kw)
    return gpu, orc


def special_keys(dtype):
    info = np.iinfo(dtype)
    ks = [0, 1, int(info.max), int(info.max) - 1]
    if info.min < 0:
        ks += [-1, int(info.min), int(info.min) + 1]
    return np.array(ks, dtype=dtype)


@pytest.mark.parametrize("key_dtype", ["int32", "uint32", "int64", "uint64"])
@pytest.mark.parametrize("dim", [1, 3, 8, 32, 64, 128])
def test_insert_then_lookup_bit_exact(key_dtype, dim):
    gpu, orc = pair([dim], key_dtype=key_dtype, opt="none")
    rng = np.random.default_rng(dim)
    info = np.iinfo(key_dtype)
    keys = np.concatenate([special_keys(key_dtype),
                           rng.integers(info.min, info.max, size=5000, dtype=key_dtype, endpoint=True)])
    keys = np.concatenate([keys, keys[::7]])  # duplicates inside one batch
    rng.shuffle(keys)
    vals, lens = gpu.lookup_or_insert(keys, dim)
    ref = orc.lookup_or_insert(keys, dim)
    np.testing.assert_array_equal(bits(vals), bits(ref))
    np.testing.assert_array_equal(lens, np.full(len(keys), dim))
    assert gpu.total_size() == orc.size() == len(np.unique(keys))
    # Lookup: present keys read their rows, absent keys read zeros.
    probe = np.concatenate([keys[:1000], rng.integers(info.min, info.max, size=1000, dtype=key_dtype)])
    got, _ = gpu.lookup(probe, dim)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(probe, dim)))


@pytest.mark.parametrize("value_dtype", ["float16", "bfloat16"])
def test_half_precision_rows(value_dtype):
    gpu, orc = pair([16, 256], key_dtype="uint64", value_dtype=value_dtype, opt="none")
    keys = splitmix64_sequence(np.arange(3000))
    for dim in (16, 256):
        vals, _ = gpu.lookup_or_insert(keys, dim)
        np.testing.assert_array_equal(bits(vals), bits(orc.lookup_or_insert(keys, dim)))
        vals, _ = gpu.lookup(keys[::-1].copy(), dim)
        np.testing.assert_array_equal(bits(vals), bits(orc.lookup(keys[::-1].copy(), dim)))


def test_cuda_tensor_path_matches_host_path():
    gpu, _ = pair([64], key_dtype="int64", opt="none")
    keys = splitmix64_sequence(np.arange(10_000)).view(np.int64)
    host_vals, _ = gpu.lookup_or_insert(keys, 64)
    dk = torch.from_numpy(keys).cuda()
    dev_vals, dev_lens = gpu.lookup(dk, 64)
    assert dev_vals.is_cuda and dev_lens.is_cuda
    np.testing.assert_array_equal(bits(dev_vals), bits(host_vals))
    dev_vals2, _ = gpu.lookup_or_insert(dk, 64)
    np.testing.assert_array_equal(bits(dev_vals2), bits(host_vals))


def test_errors():
    gpu, _ = pair([4], key_dtype="int64", opt="sgd")
    with pytest.raises(ValueError, match="key dtype does not match store"):
        gpu.lookup(np.array([1, 2], np.int32), 4)
    with pytest.raises(RuntimeError, match="invalid dim access"):
        gpu.lookup(np.array([1], np.int64), 8)
    with pytest.raises(ValueError, match="dim must be > 0"):
        gpu.lookup(np.array([1], np.int64), 0)
    with pytest.raises(ValueError, match="normalization_steps"):
        gpu.optimizer_step(normalization_steps=0)
    with pytest.raises(ValueError, match="grads shape"):
        gpu.accumulate_gradients(np.array([1, 2], np.int64), np.zeros((3, 4), np.float32))
    off = se.EmbeddingStore(se.EmbeddingConfig(dims=[4], enable_optimizer=False))
    with pytest.raises(RuntimeError, match="requires optimizer enabled"):
        off.accumulate_gradients(np.array([1], np.int64), np.zeros((1, 4), np.float32))
    with pytest.raises(RuntimeError, match="requires optimizer enabled"):
        off.optimizer_step(1)


def _train(gpu, orc, dim, steps, rng, key_pool, grad_dtype, batch=3000, absent=None, nsteps=1,
           calls_per_step=1):
    for _ in range(steps):
        for _ in range(calls_per_step):
            keys = rng.choice(key_pool, size=batch)
            vals, _ = gpu.lookup_or_insert(keys, dim)
            np.testing.assert_array_equal(bits(vals), bits(orc.lookup_or_insert(keys, dim)))
            if absent is not None:
                keys = np.concatenate([keys, absent])
            g_gpu, g_ref = make_grads((len(keys), dim), grad_dtype, rng)
            gpu.accumulate_gradients(keys, g_gpu)
            orc.accumulate_gradients(keys, g_ref, dim)
        gpu.optimizer_step(nsteps)
        orc.optimizer_step(nsteps)


def _compare_state(gpu, orc, keys, dim, nstate, exact=True):
    for k in keys:
        f1, p1, s1, t1 = gpu.read_state(int(k), dim)
        f2, p2, s2, t2 = orc.read_row(int(k), dim, nstate)
        assert f1 == f2
        if not f1:
            continue
        if exact:
            np.testing.assert_array_equal(p1, p2)
            np.testing.assert_array_equal(s1, s2)
        else:
            np.testing.assert_allclose(p1, p2, rtol=RTOL_FP32, atol=ATOL_FP32)
            np.testing.assert_allclose(s1, s2, rtol=RTOL_FP32, atol=1e-12)
        assert t1 == t2


@pytest.mark.parametrize("opt,nstate", [("sgd", 0), ("adam", 2), ("adagrad", 1)])
@pytest.mark.parametrize("dim", [1, 8, 17, 32, 64, 128])
def test_train_steps_bit_exact(opt, nstate, dim):
    okw = {"weight_decay": 0.01} if opt != "adagrad" else {"initial_accumulator_value": 0.1}
    gpu, orc = pair([dim], key_dtype="int64", opt=opt, **okw)
    rng = np.random.default_rng(100 + dim)
    pool = rng.integers(-2**63, 2**63 - 1, size=2000, dtype=np.int64)
    absent = rng.integers(-2**63, 2**63 - 1, size=50, dtype=np.int64)
    _train(gpu, orc, dim, 4, rng, pool, "float32", batch=3000, absent=absent)
    sample = np.concatenate([pool[:200], absent[:5]])
    probe, _ = gpu.lookup(pool, dim)
    np.testing.assert_array_equal(bits(probe), bits(orc.lookup(pool, dim)))
    _compare_state(gpu, orc, sample, dim, nstate)
    assert gpu.dropped_gradients() == orc.dropped() == 4 * 50


@pytest.mark.parametrize("pdt,odt,gdt", [("float16", "float32", "float16"), ("bfloat16", "bfloat16", "bfloat16"),
                                         ("float32", "float16", "bfloat16"), ("bfloat16", "float32", "float32")])
@pytest.mark.parametrize("opt", ["sgd", "adam", "adagrad"])
def test_mixed_precision_bit_exact(pdt, odt, gdt, opt):
    gpu, orc = pair([32], key_dtype="uint64", value_dtype=pdt, optimizer_dtype=odt, gradient_dtype=gdt,
                    opt=opt, gradient_scale=4.0)
    rng = np.random.default_rng(5)
    pool = splitmix64_sequence(np.arange(500))
    _train(gpu, orc, 32, 3, rng, pool, gdt, batch=1500, nsteps=2, calls_per_step=2)
    probe, _ = gpu.lookup(pool, 32)
    np.testing.assert_array_equal(bits(probe), bits(orc.lookup(pool, 32)))


def test_hot_key_long_segments_within_tolerance():
    gpu, orc = pair([64], key_dtype="int64", opt="adagrad", lr=0.01, eps=1e-8, initial_accumulator_value=0.1)
    rng = np.random.default_rng(3)
    pool = rng.integers(-2**63, 2**63 - 1, size=300, dtype=np.int64)
    hot = pool[:3]
    for _ in range(3):
        keys = np.concatenate([rng.choice(pool, size=4000), np.repeat(hot, [5000, 700, 65])])
        rng.shuffle(keys)
        gpu.lookup_or_insert(keys, 64)
        orc.lookup_or_insert(keys, 64)
        g = (rng.standard_normal((len(keys), 64)) * 1e-3).astype(np.float32)
        gpu.accumulate_gradients(keys, g)
        orc.accumulate_gradients(keys, g, 64)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    got, _ = gpu.lookup(pool, 64)
    np.testing.assert_allclose(got, orc.lookup(pool, 64), rtol=RTOL_FP32, atol=ATOL_FP32)
    _compare_state(gpu, orc, pool[:20], 64, 1, exact=False)


@pytest.mark.parametrize("dim,opt", [(64, "sgd"), (256, "adagrad"), (64, "adam")])
def test_hot_key_many_parts_and_rounds(dim, opt):
    """A key with thousands of rows packed into one stretch of the batch (its
    window holds more rows than one compaction round), spread over several
    accumulate calls; plus a moderately hot key spread over the batch.

    SGD and Adagrad parameters are compared at 1e-5. Adam divides the first
    moment by the root of the second, so an element whose summed gradient is
    near zero amplifies the summation-order difference without bound; for
    Adam the moments (linear in the sum) are compared instead."""
    okw = {"lr": 1e-3} if opt != "adagrad" else {"lr": 0.01, "initial_accumulator_value": 0.1}
    gpu, orc = pair([dim], key_dtype="uint64", opt=opt, **okw)
    rng = np.random.default_rng(17)
    pool = splitmix64_sequence(np.arange(2000))
    gpu.lookup_or_insert(pool, dim)
    orc.lookup_or_insert(pool, dim)
    for call in range(3):
        keys = rng.choice(pool, size=60_000)
        keys[10_000:13_500] = pool[0]   # 3,500 consecutive rows of one key
        keys[rng.choice(60_000, 900, replace=False)] = pool[1]
        g = (rng.standard_normal((len(keys), dim)) * 1e-3).astype(np.float32)
        gpu.accumulate_gradients(keys, g)
        orc.accumulate_gradients(keys, g, dim)
    gpu.optimizer_step(3)
    orc.optimizer_step(3)
    nstate = {"sgd": 0, "adagrad": 1, "adam": 2}[opt]
    if opt != "adam":
        got, _ = gpu.lookup(pool, dim)
        np.testing.assert_allclose(got, orc.lookup(pool, dim), rtol=RTOL_FP32, atol=ATOL_FP32)
        _compare_state(gpu, orc, pool[:8], dim, nstate, exact=False)
    else:
        for k in pool[:8]:
            f1, _, s1, t1 = gpu.read_state(int(k), dim)
            f2, _, s2, t2 = orc.read_row(int(k), dim, nstate)
            assert f1 and f2 and t1 == t2 == 1
            # normwise: |dm| <= 1e-5 * max|m| (a near-zero sum has no relative accuracy)
            for a, b in ((s1[:dim], s2[:dim]), (s1[dim:], s2[dim:])):
                np.testing.assert_allclose(a, b, rtol=RTOL_FP32, atol=RTOL_FP32 * np.abs(b).max())


def test_gradient_overflow_rejected_and_not_accumulated():
    # test_mixed_precision.py:457-472
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[1], value_dtype="float16", optimizer_dtype="float32",
                                               gradient_dtype="float32", key_dtype="uint64"),
                            optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    key = np.array([1], dtype=np.uint64)
    gpu.lookup_or_insert(key, 1)
    with pytest.raises((OverflowError, ValueError), match="gradient"):
        gpu.accumulate_gradients(key, np.array([[100000.0]], dtype=np.float32))
    gpu.accumulate_gradients(key, np.array([[2.0]], dtype=np.float32))
    gpu.optimizer_step(1)
    vals, _ = gpu.lookup(key, 1)
    np.testing.assert_array_equal(np.asarray(vals).astype(np.float32), [-2.0])


def test_device_gradient_overflow_poisons_window():
    """CUDA gradient inputs are validated on the device without a stall: a
    failing batch discards its accumulation window and the OverflowError is
    raised by the next synchronising call; training then continues."""
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[4], value_dtype="float16", optimizer_dtype="float32",
                                               gradient_dtype="float32", key_dtype="int64"),
                            optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    keys = torch.tensor([1, 2], dtype=torch.int64, device="cuda")
    gpu.lookup_or_insert(keys, 4)
    gpu.accumulate_gradients(keys, torch.ones((2, 4), device="cuda"))
    gpu.accumulate_gradients(keys, torch.full((2, 4), 1e6, device="cuda"))  # above float16 range
    gpu.optimizer_step(1)
    with pytest.raises(OverflowError, match="gradient"):
        gpu.synchronize()
    vals, _ = gpu.lookup(keys, 4)
    assert torch.equal(vals.cpu().float(), torch.zeros(8))  # the whole window was discarded
    gpu.accumulate_gradients(keys, torch.ones((2, 4), device="cuda"))
    gpu.optimizer_step(1)
    gpu.synchronize()
    vals, _ = gpu.lookup(keys, 4)
    assert torch.equal(vals.cpu().float(), -torch.ones(8))


@pytest.mark.parametrize("n", [1, 2, 3])
@pytest.mark.parametrize("scale,gdt", [(1.0, "float32"), (8.0, "float16")])
def test_normalization_window(n, scale, gdt):
    # test_mixed_precision.py:408-438
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[1], value_dtype="float32", optimizer_dtype="float32",
                                               gradient_dtype=gdt, gradient_scale=scale, key_dtype="int64"),
                            optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    keys = np.asarray([17], dtype=np.int64)
    gpu.lookup_or_insert(keys, 1)
    for _ in range(n):
        gpu.accumulate_gradients(keys, np.asarray([[3.0]], dtype=np.dtype(gdt)))
    gpu.optimizer_step(normalization_steps=n)
    vals, _ = gpu.lookup(keys, 1)
    np.testing.assert_allclose(np.asarray(vals), [-3.0], atol=2e-3)


def test_reference_store_tests():
    # hogwild_storage_test.cpp:42-103: SGD normalized update == -lr/2 within 1e-6.
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[8], key_dtype="int64"), optimizer_config=se.Sgd(lr=1.0),
                            initializer_config=se.Zeros())
    keys = np.arange(4096, dtype=np.int64)
    gpu.lookup_or_insert(keys, 8)
    gpu.accumulate_gradients(keys, np.ones((4096, 8), np.float32))
    gpu.optimizer_step(2)
    np.testing.assert_allclose(np.asarray(gpu.lookup(keys, 8)[0]), -0.5, atol=1e-6)
    # test_embedding_table.py:279-316: per-ID Adam step.
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[128], key_dtype="uint64"), initializer_config=se.Zeros(),
                            optimizer_config=se.Adam(lr=0.001))
    k0, k1 = np.array([0], np.uint64), np.array([1], np.uint64)
    g = np.ones((1, 128), np.float32)
    gpu.lookup_or_insert(k0, 128)
    gpu.accumulate_gradients(k0, g)
    gpu.optimizer_step(1)
    v0 = np.asarray(gpu.lookup(k0, 128)[0]).copy()
    for _ in range(100):
        gpu.accumulate_gradients(k0, g)
        gpu.optimizer_step(1)
    gpu.lookup_or_insert(k1, 128)
    gpu.accumulate_gradients(k1, g)
    gpu.optimizer_step(1)
    np.testing.assert_allclose(v0, np.asarray(gpu.lookup(k1, 128)[0]), atol=1e-6)
    assert gpu.read_state(0, 128)[3] == 101 and gpu.read_state(1, 128)[3] == 1
    # test_collision_accumulation.py: hot keys move negative under repeated accumulation.
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[16], thread_budget=2), initializer_config=se.Zeros(),
                            optimizer_config=se.Adam(lr=0.01))
    keys = np.array([101, 102], np.int64)
    gpu.lookup_or_insert(keys, 16)
    for _ in range(4):
        gpu.accumulate_gradients(keys, np.ones((2, 16), np.float32) * 0.1)
    gpu.optimizer_step(1)
    v1 = np.asarray(gpu.lookup(keys, 16)[0]).copy()
    assert np.all(v1 < 0)
    for _ in range(4):
        gpu.accumulate_gradients(keys, np.ones((2, 16), np.float32) * 0.1)
    gpu.optimizer_step(1)
    assert np.all(np.asarray(gpu.lookup(keys, 16)[0]) < v1)


def test_growth_beyond_initial_capacity():
    gpu, orc = pair([8], key_dtype="int64", opt="adam", capacity=64)
    keys = np.arange(50_000, dtype=np.int64) * 7919
    for chunk in np.array_split(keys, 7):
        vals, _ = gpu.lookup_or_insert(chunk, 8)
        np.testing.assert_array_equal(bits(vals), bits(orc.lookup_or_insert(chunk, 8)))
    assert gpu.total_size() == 50_000
    got, _ = gpu.lookup(keys, 8)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(keys, 8)))
    gpu.reserve(200_000, 8)
    got, _ = gpu.lookup(keys, 8)
    np.testing.assert_array_equal(bits(got), bits(orc.lookup(keys, 8)))


def test_train_workload_small_scale_parity():
    """The train-step workload (Zipf 1.05 + 5% new keys, Adagrad) at a size the
    oracle handles in seconds: 200k warmed keys, 4 steps of 65,536 keys."""
    wl = TrainWorkload(num_keys=200_000, batch=65_536)
    gpu, orc = pair([64], key_dtype="int64", opt="adagrad", lr=0.01, eps=1e-8, initial_accumulator_value=0.1,
                    capacity=300_000)
    warm = wl.warm_keys()
    gpu.lookup_or_insert(warm, 64)
    orc.lookup_or_insert(warm, 64)
    keys, grads = wl.make_batches(4)
    for s in range(4):
        vals, _ = gpu.lookup_or_insert(keys[s], 64)
        ref = orc.lookup_or_insert(keys[s], 64)
        if s == 0:  # before any update every row is its initializer output
            np.testing.assert_array_equal(bits(vals), bits(ref))
        else:  # hot keys (> 64 rows per step) are reduced in parallel runs
            np.testing.assert_allclose(vals, ref, rtol=RTOL_FP32, atol=ATOL_FP32)
        gpu.accumulate_gradients(keys[s], grads[s])
        orc.accumulate_gradients(keys[s], grads[s], 64)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    touched = np.unique(keys)
    got, _ = gpu.lookup(touched, 64)
    np.testing.assert_allclose(got, orc.lookup(touched, 64), rtol=RTOL_FP32, atol=ATOL_FP32)
    assert gpu.total_size() == orc.size()


def test_growth_between_accumulate_and_step():
    """Rows are counted for the step when gradients are appended; an arena
    and pending-buffer growth before the step must keep those counts."""
    gpu, orc = pair([16], key_dtype="int64", opt="adagrad", lr=0.01, eps=1e-8, initial_accumulator_value=0.1,
                    capacity=64)
    rng = np.random.default_rng(11)
    a = rng.integers(-2**62, 2**62, size=200, dtype=np.int64)
    hot = np.repeat(a[:5], 40)  # a few keys with many rows
    keys = np.concatenate([a, hot])
    gpu.lookup_or_insert(keys, 16)
    orc.lookup_or_insert(keys, 16)
    g = (rng.standard_normal((len(keys), 16)) * 1e-2).astype(np.float32)
    gpu.accumulate_gradients(keys, g)
    orc.accumulate_gradients(keys, g, 16)
    # grow the arena (and the directory) before the step
    b = rng.integers(-2**62, 2**62, size=20_000, dtype=np.int64)
    gpu.lookup_or_insert(b, 16)
    orc.lookup_or_insert(b, 16)
    # and the pending buffers
    g2 = (rng.standard_normal((len(b), 16)) * 1e-2).astype(np.float32)
    gpu.accumulate_gradients(b, g2)
    orc.accumulate_gradients(b, g2, 16)
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    probe = np.concatenate([a, b])
    got, _ = gpu.lookup(probe, 16)
    np.testing.assert_allclose(np.asarray(got), orc.lookup(probe, 16).reshape(np.asarray(got).shape),
                               rtol=RTOL_FP32, atol=ATOL_FP32)


def test_large_window_sorted_placement():
    """More pending rows than one hot-key window (131,072): segments are laid
    out by a stable sort. Thousands of keys with 65..5,000 rows; results
    within the fp32 tolerance of the oracle's serial sums and identical, bit
    for bit, between two stores fed the same calls."""
    from sparse_embedding_b200.workloads import Zipf

    dim = 32
    gpu, orc = pair([dim], key_dtype="uint64", opt="adagrad", lr=0.01, initial_accumulator_value=0.1)
    twin, _ = pair([dim], key_dtype="uint64", opt="adagrad", lr=0.01, initial_accumulator_value=0.1)
    rng = np.random.default_rng(23)
    pool = splitmix64_sequence(np.arange(50_000))
    z = Zipf(len(pool), 1.1, 5)
    for step in range(2):
        keys = pool[z.sample(rng, 300_000)]
        g = (rng.standard_normal((len(keys), dim)) * 1e-3).astype(np.float32)
        for s in (gpu, twin):
            s.lookup_or_insert(keys, dim)
            s.accumulate_gradients(keys, g)
            s.optimizer_step(1)
        orc.lookup_or_insert(keys, dim)
        orc.accumulate_gradients(keys, g, dim)
        orc.optimizer_step(1)
    got, _ = gpu.lookup(pool, dim)
    np.testing.assert_allclose(got, orc.lookup(pool, dim), rtol=RTOL_FP32, atol=ATOL_FP32)
    np.testing.assert_array_equal(bits(got), bits(twin.lookup(pool, dim)[0]))


@pytest.mark.parametrize("gather", ["vector", "bulk"])
@pytest.mark.parametrize("dim,value_dtype", [(128, "float32"), (256, "bfloat16"), (200, "float32"),
                                             (256, "float32"), (400, "float16"), (129, "float32")])
def test_wide_row_lookup_bit_exact(dim, value_dtype, gather, monkeypatch):
    """forward_lookup of rows of 512..1,024 bytes: the default vector-load
    gather, and the TMA bulk kernel (SE_GPU_WIDE_GATHER=bulk: bulk copies
    per row into shared memory, one bulk store per 32 positions); a 516-byte
    row (dim 129 fp32) always takes the vector path. Absent keys read as
    zeros; batches not a multiple of 32; device and host outputs."""
    if gather == "bulk":
        monkeypatch.setenv("SE_GPU_WIDE_GATHER", "bulk")
    else:
        monkeypatch.delenv("SE_GPU_WIDE_GATHER", raising=False)
    gpu, orc = pair([dim], key_dtype="int64", value_dtype=value_dtype, opt="none")
    rng = np.random.default_rng(dim)
    present = rng.integers(-2**63, 2**63 - 1, size=3000, dtype=np.int64)
    gpu.lookup_or_insert(present, dim)
    orc.lookup_or_insert(present, dim)
    absent = rng.integers(-2**63, 2**63 - 1, size=500, dtype=np.int64)
    gpu.profile(True)
    gpu.lookup(present[:64], dim)
    _, bulk_launches = gpu.profile_read("k_lookup_bulk")
    gpu.profile(False)
    row_bytes = dim * (4 if value_dtype == "float32" else 2)
    eligible = 512 <= row_bytes <= 1024 and row_bytes % 16 == 0
    assert bulk_launches == (1 if gather == "bulk" and eligible else 0)
    for n in (1, 31, 33, 1000, 3457):
        keys = rng.choice(np.concatenate([present, absent]), size=n)
        want = orc.lookup(keys, dim)
        got, lens = gpu.lookup(keys, dim)
        np.testing.assert_array_equal(bits(got).ravel(), bits(want).ravel())
        assert np.all(np.asarray(lens) == dim)
        dev, dlens = gpu.lookup(torch.from_numpy(keys).cuda(), dim)
        np.testing.assert_array_equal(bits(dev).ravel(), bits(want).ravel())
        assert int(dlens.min()) == dim and dlens.shape == (n,)
