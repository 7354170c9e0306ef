"""Atomic accumulation mode on the GPU against the CPU oracle, through the C ABI (GPU).

In atomic mode gradient rows are added into per-key fp32 sums as they arrive
(red.global.add.v4.f32), so a key's rows are not summed in arrival order.
Forward gathers and inserted rows stay bit-identical to the oracle; updates
are compared at the tolerances below:
  fp32 tables: 1e-5 relative (atol 1e-5 of the values' 0.05 scale);
  fp16 / bf16 parameters: one unit in the last place of the stored dtype
  (the ordered sum rounds to the gradient dtype after every add, the atomic
  sum only once).
Adam divides the first moment by the root of the second, which amplifies
the reassociation error of a sum that cancels to near zero without bound,
so Adam runs use gradients of one sign (no cancellation) or compare the
moments, which are linear in the sum.
"""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from oracle import oracle as O
from sparse_embedding_b200.workloads import TrainWorkload, splitmix64_sequence

pytestmark = pytest.mark.gpu

RTOL_FP32 = 1e-5
ATOL_FP32 = RTOL_FP32 * 0.05
RTOL_HALF = {"float16": 2e-3, "bfloat16": 1e-2}


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


def as_f32(x, dtype="float32"):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().float().numpy()
    x = np.asarray(x)
    if dtype == "bfloat16" and x.dtype == np.uint16:
        return (x.astype(np.uint32) << 16).view(np.float32)
    if x.dtype == np.uint16:
        return x.view(np.float16).astype(np.float32)
    return x.astype(np.float32)


def pair(dims, key_dtype="int64", value_dtype="float32", optimizer_dtype="", gradient_dtype="",
         gradient_scale=1.0, init="uniform", opt="adagrad", capacity=0, **okw):
    cfg = se.EmbeddingConfig(dims=dims, thread_budget=1, key_dtype=key_dtype, value_dtype=value_dtype,
                             optimizer_dtype=optimizer_dtype, gradient_dtype=gradient_dtype,
                             gradient_scale=gradient_scale, enable_optimizer=opt != "none",
                             initial_capacity=capacity, accumulation="atomic")
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


def grads_for(shape, rng, positive=False, scale=1e-2):
    g = rng.standard_normal(shape) * scale
    if positive:
        g = np.abs(g) + 0.1 * scale
    return g.astype(np.float32)


def compare_rows(gpu, orc, keys, dim):
    got, _ = gpu.lookup(keys, dim)
    np.testing.assert_allclose(np.asarray(got), orc.lookup(keys, dim), rtol=RTOL_FP32, atol=ATOL_FP32)


def compare_state(gpu, orc, keys, dim, nstate):
    for k in keys:
        f1, p1, s1, t1 = gpu.read_state(int(k), dim)
        f2, p2, s2, t2 = orc.read_row(int(k), dim, nstate)
        assert f1 == f2
        if not f1:
            continue
        np.testing.assert_allclose(p1, p2, rtol=RTOL_FP32, atol=ATOL_FP32)
        if nstate:
            np.testing.assert_allclose(s1, s2, rtol=RTOL_FP32, atol=RTOL_FP32 * np.abs(s2).max())
        assert t1 == t2


@pytest.mark.parametrize("opt,nstate", [("sgd", 0), ("adam", 2), ("adagrad", 1)])
@pytest.mark.parametrize("dim", [1, 8, 17, 32, 64, 128, 256])
def test_train_steps_within_tolerance(opt, nstate, dim):
    okw = {"weight_decay": 0.01} if opt != "adagrad" else {"initial_accumulator_value": 0.1}
    gpu, orc = pair([dim], key_dtype="int64", opt=opt, **okw)
    rng = np.random.default_rng(200 + dim)
    pool = rng.integers(-2**63, 2**63 - 1, size=2000, dtype=np.int64)
    absent = rng.integers(-2**63, 2**63 - 1, size=50, dtype=np.int64)
    for _ in range(4):
        keys = rng.choice(pool, size=3000)
        vals, _ = gpu.lookup_or_insert(keys, dim)
        ref = orc.lookup_or_insert(keys, dim)
        np.testing.assert_allclose(np.asarray(vals), ref, rtol=RTOL_FP32, atol=ATOL_FP32)
        keys = np.concatenate([keys, absent])
        g = grads_for((len(keys), dim), rng, positive=opt == "adam")
        gpu.accumulate_gradients(keys, g)
        orc.accumulate_gradients(keys, g, dim)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    compare_rows(gpu, orc, pool, dim)
    compare_state(gpu, orc, np.concatenate([pool[:100], absent[:5]]), dim, nstate)
    assert gpu.dropped_gradients() == orc.dropped() == 4 * 50


def test_single_rows_bit_exact():
    """With at most two rows per key and window the sum has one rounding in
    either order, so the update equals the ordered mode bit for bit."""
    gpu, orc = pair([64], key_dtype="uint64", opt="adagrad", lr=0.01, initial_accumulator_value=0.1)
    rng = np.random.default_rng(1)
    pool = splitmix64_sequence(np.arange(5000))
    for _ in range(3):
        keys = np.concatenate([pool, pool[:1000]])
        rng.shuffle(keys)
        np.testing.assert_array_equal(bits(gpu.lookup_or_insert(keys, 64)[0]), bits(orc.lookup_or_insert(keys, 64)))
        g = grads_for((len(keys), 64), rng)
        gpu.accumulate_gradients(keys, g)
        orc.accumulate_gradients(keys, g, 64)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    np.testing.assert_array_equal(bits(gpu.lookup(pool, 64)[0]), bits(orc.lookup(pool, 64)))


@pytest.mark.parametrize("pdt,odt,gdt", [("float16", "float32", "float16"), ("bfloat16", "bfloat16", "bfloat16"),
                                         ("float32", "float16", "bfloat16"), ("bfloat16", "float32", "float32")])
@pytest.mark.parametrize("opt", ["sgd", "adagrad"])
def test_mixed_precision_within_tolerance(pdt, odt, gdt, opt):
    gpu, orc = pair([32], key_dtype="uint64", value_dtype=pdt, optimizer_dtype=odt, gradient_dtype=gdt,
                    opt=opt, gradient_scale=4.0)
    rng = np.random.default_rng(5)
    pool = splitmix64_sequence(np.arange(500))
    for step in range(3):
        for _ in range(2):
            keys = rng.choice(pool, size=1500)
            vals, _ = gpu.lookup_or_insert(keys, 32)
            ref = orc.lookup_or_insert(keys, 32)
            if step == 0:  # before any update every row is its initializer output
                np.testing.assert_array_equal(bits(vals), bits(ref))
            g = grads_for((len(keys), 32), rng)
            if gdt == "float32":
                g_gpu, g_ref = g, g
            elif gdt == "float16":
                g_gpu = g.astype(np.float16)
                g_ref = g_gpu.view(np.uint16)
            else:
                g_gpu = torch.from_numpy(g).to(torch.bfloat16)
                g_ref = bits(g_gpu)
            gpu.accumulate_gradients(keys, g_gpu)
            orc.accumulate_gradients(keys, g_ref, 32)
        gpu.optimizer_step(2)
        orc.optimizer_step(2)
    got = as_f32(gpu.lookup(pool, 32)[0])
    ref = as_f32(orc.lookup(pool, 32), pdt)
    # the coarser of the parameter and the gradient dtype bounds the difference
    rtol = max(RTOL_HALF.get(pdt, RTOL_FP32), RTOL_HALF.get(gdt, RTOL_FP32))
    np.testing.assert_allclose(got.reshape(ref.shape), ref, rtol=rtol, atol=rtol * 0.05)


@pytest.mark.parametrize("dim,opt", [(64, "sgd"), (256, "adagrad"), (64, "adam"), (20, "adagrad")])
def test_hot_keys(dim, opt):
    """Keys with thousands of rows in one window, spread over several calls
    and packed into runs: every tile of the batch adds its own sum."""
    okw = {"lr": 1e-3} if opt != "adagrad" else {"lr": 0.01, "initial_accumulator_value": 0.1}
    gpu, orc = pair([dim], key_dtype="uint64", opt=opt, **okw)
    rng = np.random.default_rng(17)
    pool = splitmix64_sequence(np.arange(2000))
    gpu.lookup_or_insert(pool, dim)
    orc.lookup_or_insert(pool, dim)
    for _ in range(3):
        keys = rng.choice(pool, size=60_000)
        keys[10_000:13_500] = pool[0]
        keys[rng.choice(60_000, 900, replace=False)] = pool[1]
        g = grads_for((len(keys), dim), rng, scale=1e-3)
        gpu.accumulate_gradients(keys, g)
        orc.accumulate_gradients(keys, g, dim)
    gpu.optimizer_step(3)
    orc.optimizer_step(3)
    nstate = {"sgd": 0, "adagrad": 1, "adam": 2}[opt]
    if opt != "adam":
        compare_rows(gpu, orc, pool, dim)
        compare_state(gpu, orc, pool[:8], dim, nstate)
    else:
        for k in pool[:8]:
            f1, _, s1, t1 = gpu.read_state(int(k), dim)
            f2, _, s2, t2 = orc.read_row(int(k), dim, nstate)
            assert f1 and f2 and t1 == t2 == 1
            for a, b in ((s1[:dim], s2[:dim]), (s1[dim:], s2[dim:])):
                np.testing.assert_allclose(a, b, rtol=RTOL_FP32, atol=RTOL_FP32 * np.abs(b).max())


def test_special_keys_and_absent_then_inserted():
    """The all-ones key and key 0 are ordinary keys; a key absent when its
    gradients arrive but inserted before optimizer_step receives them (keys
    are resolved at step time, like the reference's transient arena); a key
    erased before the step drops its rows."""
    gpu, orc = pair([16], key_dtype="uint64", opt="sgd", lr=1.0, init="zeros")
    keys = np.array([2**64 - 1, 0, 5, 2**64 - 1, 7], dtype=np.uint64)
    late = np.array([11, 12], dtype=np.uint64)
    gpu.lookup_or_insert(keys, 16)
    orc.lookup_or_insert(keys, 16)
    both = np.concatenate([keys, late])
    g = np.arange(len(both) * 16, dtype=np.float32).reshape(len(both), 16) / 64.0
    gpu.accumulate_gradients(both, g)
    orc.accumulate_gradients(both, g, 16)
    gpu.lookup_or_insert(late[:1], 16)   # key 11 arrives after its gradient
    orc.lookup_or_insert(late[:1], 16)
    gpu.erase(np.array([7], dtype=np.uint64))
    orc.erase(np.array([7], dtype=np.uint64))
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    probe = np.array([2**64 - 1, 0, 5, 7, 11, 12], dtype=np.uint64)
    np.testing.assert_array_equal(bits(gpu.lookup(probe, 16)[0]), bits(orc.lookup(probe, 16)))
    assert gpu.dropped_gradients() == orc.dropped() == 2  # key 12 (never inserted) and erased key 7


def test_gradient_overflow_rejected_and_not_accumulated():
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[1], value_dtype="float16", optimizer_dtype="float32",
                                               gradient_dtype="float32", key_dtype="uint64",
                                               accumulation="atomic"),
                            optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    key = np.array([1], dtype=np.uint64)
    gpu.lookup_or_insert(key, 1)
    with pytest.raises(OverflowError, match="gradient"):
        gpu.accumulate_gradients(key, np.array([[100000.0]], dtype=np.float32))
    gpu.accumulate_gradients(key, np.array([[2.0]], dtype=np.float32))
    gpu.optimizer_step(1)
    vals, _ = gpu.lookup(key, 1)
    np.testing.assert_array_equal(np.asarray(vals).astype(np.float32), [-2.0])


def test_device_gradient_overflow_poisons_window():
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[4], value_dtype="float16", optimizer_dtype="float32",
                                               gradient_dtype="float32", key_dtype="int64",
                                               accumulation="atomic"),
                            optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    keys = torch.tensor([1, 2], dtype=torch.int64, device="cuda")
    gpu.lookup_or_insert(keys, 4)
    gpu.accumulate_gradients(keys, torch.ones((2, 4), device="cuda"))
    gpu.accumulate_gradients(keys, torch.full((2, 4), 1e6, device="cuda"))
    gpu.optimizer_step(1)
    with pytest.raises(OverflowError, match="gradient"):
        gpu.synchronize()
    vals, _ = gpu.lookup(keys, 4)
    assert torch.equal(vals.cpu().float(), torch.zeros(8))
    gpu.accumulate_gradients(keys, torch.ones((2, 4), device="cuda"))
    gpu.optimizer_step(1)
    gpu.synchronize()
    vals, _ = gpu.lookup(keys, 4)
    assert torch.equal(vals.cpu().float(), -torch.ones(8))


@pytest.mark.parametrize("n", [1, 2, 3])
@pytest.mark.parametrize("scale,gdt", [(1.0, "float32"), (8.0, "float16")])
def test_normalization_window(n, scale, gdt):
    gpu = se.EmbeddingStore(se.EmbeddingConfig(dims=[1], value_dtype="float32", optimizer_dtype="float32",
                                               gradient_dtype=gdt, gradient_scale=scale, key_dtype="int64",
                                               accumulation="atomic"),
                            optimizer_config=se.Sgd(lr=1.0), initializer_config=se.Zeros())
    keys = np.asarray([17], dtype=np.int64)
    gpu.lookup_or_insert(keys, 1)
    for _ in range(n):
        gpu.accumulate_gradients(keys, np.asarray([[3.0]], dtype=np.dtype(gdt)))
    gpu.optimizer_step(normalization_steps=n)
    vals, _ = gpu.lookup(keys, 1)
    np.testing.assert_allclose(np.asarray(vals), [-3.0], atol=2e-3)


def test_window_outgrows_sum_table_and_arena():
    """Several accumulate calls in one window: the sum table grows between
    them (claimed slots move to the larger table), and the arena and the
    directory grow between accumulate and step."""
    gpu, orc = pair([16], key_dtype="int64", opt="adagrad", lr=0.01, initial_accumulator_value=0.1, capacity=64)
    rng = np.random.default_rng(11)
    a = rng.integers(-2**62, 2**62, size=200, dtype=np.int64)
    keys = np.concatenate([a, np.repeat(a[:5], 40)])
    gpu.lookup_or_insert(keys, 16)
    orc.lookup_or_insert(keys, 16)
    g = grads_for((len(keys), 16), rng)
    gpu.accumulate_gradients(keys, g)
    orc.accumulate_gradients(keys, g, 16)
    b = rng.integers(-2**62, 2**62, size=20_000, dtype=np.int64)
    gpu.lookup_or_insert(b, 16)
    orc.lookup_or_insert(b, 16)
    for part in np.array_split(np.concatenate([b, a]), 3):
        g2 = grads_for((len(part), 16), rng)
        gpu.accumulate_gradients(part, g2)
        orc.accumulate_gradients(part, g2, 16)
    gpu.optimizer_step(1)
    orc.optimizer_step(1)
    compare_rows(gpu, orc, np.concatenate([a, b]), 16)


def test_embedding_bag_backward():
    """The bag backward accumulates each bag's gradient for every key of the
    bag; in atomic mode it equals accumulating the expanded rows."""
    dim = 32
    cfg = dict(dims=[dim], key_dtype="int64", accumulation="atomic")
    bag = se.EmbeddingStore(se.EmbeddingConfig(**cfg), optimizer_config=se.Sgd(lr=0.5))
    flat, orc = pair([dim], key_dtype="int64", opt="sgd", lr=0.5)
    rng = np.random.default_rng(4)
    pool = rng.integers(-2**62, 2**62, size=300, dtype=np.int64)
    sizes = rng.integers(1, 12, size=400)
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    keys = rng.choice(pool, size=int(offsets[-1]))
    pooled_g = grads_for((len(sizes), dim), rng)
    bag.embedding_bag(keys, offsets, dim, insert=True)
    bag.embedding_bag_backward(keys, offsets, pooled_g)
    bag.optimizer_step(1)
    flat.lookup_or_insert(keys, dim)
    orc.lookup_or_insert(keys, dim)
    expanded = np.repeat(pooled_g, sizes, axis=0)
    flat.accumulate_gradients(keys, expanded)
    orc.accumulate_gradients(keys, expanded, dim)
    flat.optimizer_step(1)
    orc.optimizer_step(1)
    got = np.asarray(bag.lookup(pool, dim)[0])
    np.testing.assert_allclose(got, np.asarray(flat.lookup(pool, dim)[0]), rtol=RTOL_FP32, atol=ATOL_FP32)
    np.testing.assert_allclose(got, orc.lookup(pool, dim), rtol=RTOL_FP32, atol=ATOL_FP32)


def test_train_workload_small_scale_parity():
    """The train-step workload (Zipf 1.05 + 5% new keys, Adagrad) at a size the
    oracle handles in seconds: 200k warmed keys, 4 steps of 65,536 keys, with
    device-resident inputs (the path the benchmark times)."""
    wl = TrainWorkload(num_keys=200_000, batch=65_536)
    gpu, orc = pair([64], key_dtype="int64", opt="adagrad", lr=0.01, eps=1e-8, initial_accumulator_value=0.1,
                    capacity=300_000)
    warm = wl.warm_keys()
    gpu.lookup_or_insert(torch.from_numpy(warm).cuda(), 64)
    orc.lookup_or_insert(warm, 64)
    keys, grads = wl.make_batches(4)
    for s in range(4):
        k = torch.from_numpy(keys[s]).cuda()
        vals, _ = gpu.lookup_or_insert(k, 64)
        ref = orc.lookup_or_insert(keys[s], 64)
        np.testing.assert_allclose(vals.cpu().numpy(), ref, rtol=RTOL_FP32, atol=ATOL_FP32)
        gpu.accumulate_gradients(k, torch.from_numpy(grads[s]).cuda())
        orc.accumulate_gradients(keys[s], grads[s], 64)
        gpu.optimizer_step(1)
        orc.optimizer_step(1)
    touched = np.unique(keys)
    compare_rows(gpu, orc, touched, 64)
    assert gpu.total_size() == orc.size()


def test_graph_replay_matches_eager():
    """The train step captured in a CUDA graph and replayed gives the same
    rows as the same calls run eagerly on a twin store."""
    dim = 64
    wl = TrainWorkload(num_keys=50_000, batch=8192)
    stores = [pair([dim], key_dtype="int64", opt="adagrad", lr=0.01, initial_accumulator_value=0.1,
                   capacity=200_000)[0] for _ in range(2)]
    warm = torch.from_numpy(wl.warm_keys()).cuda()
    keys, grads = wl.make_batches(4)
    kd = torch.from_numpy(keys).cuda()
    gd = torch.from_numpy(grads).cuda()
    for st in stores:
        st.lookup_or_insert(warm, dim)
        st.lookup_or_insert(kd[0], dim)
        st.accumulate_gradients(kd[0], gd[0])
        st.optimizer_step(1)
    torch.cuda.synchronize()
    graph_store, eager_store = stores
    kbuf, gbuf = kd[1].clone(), gd[1].clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        graph_store.lookup_or_insert(kbuf, dim)
        graph_store.accumulate_gradients(kbuf, gbuf)
        graph_store.optimizer_step(1)
    for s in range(1, 4):
        kbuf.copy_(kd[s])
        gbuf.copy_(gd[s])
        g.replay()
        eager_store.lookup_or_insert(kd[s], dim)
        eager_store.accumulate_gradients(kd[s], gd[s])
        eager_store.optimizer_step(1)
    torch.cuda.synchronize()
    touched = torch.unique(kd)
    a = graph_store.lookup(touched, dim)[0].cpu().numpy()
    b = eager_store.lookup(touched, dim)[0].cpu().numpy()
    np.testing.assert_allclose(a, b, rtol=RTOL_FP32, atol=ATOL_FP32)
