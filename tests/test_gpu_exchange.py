"""Peer-memory exchange kernels on one GPU, through the C ABI.

With one rank the exchange runs its whole pipeline (route, publish, scatter
into the inbox, owner insert / gather into the row buffer, row return,
gradient scatter and accumulate) against its own arena, so its results must
equal the oracle store's bit for bit. The timeout case connects two ranks'
ends in this process and drives only rank 0: its waits for rank 1's flags,
which nothing sets, must give up after the exchange's timeout and report it,
leaving the CUDA context usable.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from sparse_embedding_b200 import _native as N

pytestmark = pytest.mark.gpu
DIM = 32


def _store(key_dtype="int64"):
    import sparse_embedding_b200 as se

    return se.EmbeddingStore(se.EmbeddingConfig(dims=[DIM], key_dtype=key_dtype, device=0),
                             optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))


def _exchange(store, world, rank, max_keys, timeout_ms=20_000, kind="hash"):
    h = C.c_void_p()
    N.check(N.lib().se_exchange_create(store._h, N.PART_CODES[kind], world, rank, max_keys, DIM, timeout_ms,
                                       C.byref(h)))
    return h


def _connect_local(handles):
    arr = (C.c_void_p * len(handles))(*[h.value for h in handles])
    N.check(N.lib().se_exchange_connect_local(arr, len(handles)))


@pytest.mark.parametrize("key_dtype", ["int64", "int32"])
def test_single_rank_exchange_matches_oracle(key_dtype):
    from oracle import oracle as O

    L = N.lib()
    torch.cuda.set_device(0)
    store = _store(key_dtype)
    ex = _exchange(store, 1, 0, 4096)
    _connect_local([ex])
    single = O.OracleStore([DIM], key_dtype=key_dtype, optimizer="adagrad", lr=0.01, eps=1e-8,
                           initial_accumulator=0.1)
    rng = np.random.default_rng(5)
    info = np.iinfo(np.int64 if key_dtype == "int64" else np.int32)
    pool = rng.integers(info.min, info.max, size=700, dtype=info.dtype)
    st = torch.cuda.current_stream().cuda_stream
    for step in range(4):
        keys = np.concatenate([rng.choice(pool, size=3000), rng.integers(info.min, info.max, size=50,
                                                                          dtype=info.dtype)])
        grads = (rng.standard_normal((len(keys), DIM)) * 1e-2).astype(np.float32)
        k = torch.from_numpy(keys).cuda()
        out = torch.empty((len(keys), DIM), dtype=torch.float32, device="cuda")
        N.check(L.se_exchange_lookup(ex, k.data_ptr(), len(keys), out.data_ptr(), 1, C.c_void_p(st)))
        want = single.lookup_or_insert(keys, DIM)
        np.testing.assert_array_equal(out.cpu().numpy().ravel().view(np.uint32), want.view(np.uint32))
        g = torch.from_numpy(grads).cuda()
        if step % 2:
            N.check(L.se_exchange_accumulate(ex, k.data_ptr(), len(keys), g.data_ptr(), C.c_void_p(st)))
        else:  # rows routed like the lookup's keys
            N.check(L.se_exchange_accumulate_routed(ex, g.data_ptr(), len(keys), C.c_void_p(st)))
        single.accumulate_gradients(keys, grads, DIM)
        store.optimizer_step(1)
        single.optimizer_step(1)
        N.check(L.se_exchange_check(ex, C.c_void_p(st)))
    probe = np.concatenate([pool, rng.integers(info.min, info.max, size=30, dtype=info.dtype)])
    pk = torch.from_numpy(probe).cuda()
    out = torch.empty((len(probe), DIM), dtype=torch.float32, device="cuda")
    N.check(L.se_exchange_lookup(ex, pk.data_ptr(), len(probe), out.data_ptr(), 0, C.c_void_p(st)))
    want = single.lookup(probe, DIM)
    np.testing.assert_array_equal(out.cpu().numpy().ravel().view(np.uint32), want.view(np.uint32))
    N.check(L.se_exchange_check(ex, C.c_void_p(st)))
    N.check(L.se_exchange_destroy(ex))


@pytest.mark.parametrize("accumulation", ["ordered", "atomic"])
@pytest.mark.parametrize("key_dtype", ["int64", "int32"])
def test_single_rank_exchange_dedupe(key_dtype, accumulation):
    """Sender-side dedupe on one rank: every distinct key of the batch is
    routed once and the rows expanded to the batch's positions - identical to
    the oracle bit for bit (the all-ones / -1 key included); the routed
    gradients are summed per key on the sender first, so updates match
    within 1e-5 relative (atol 1e-5 of the values' 0.05 scale). Keyed
    gradient batches (not routed like the lookup) keep the plain route."""
    import sparse_embedding_b200 as se
    from oracle import oracle as O

    L = N.lib()
    torch.cuda.set_device(0)
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[DIM], key_dtype=key_dtype, device=0,
                                                 accumulation=accumulation),
                              optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))
    ex = _exchange(store, 1, 0, 8192)
    N.check(L.se_exchange_set_dedupe(ex, 1))
    _connect_local([ex])
    single = O.OracleStore([DIM], key_dtype=key_dtype, optimizer="adagrad", lr=0.01, eps=1e-8,
                           initial_accumulator=0.1)
    rng = np.random.default_rng(9)
    info = np.iinfo(np.int64 if key_dtype == "int64" else np.int32)
    pool = np.concatenate([rng.integers(info.min, info.max, size=700, dtype=info.dtype),
                           np.array([-1, 0], dtype=info.dtype)])
    st = torch.cuda.current_stream().cuda_stream
    for step in range(5):
        keys = np.concatenate([rng.choice(pool, size=5000), np.repeat(pool[:2], 900),
                               rng.integers(info.min, info.max, size=50, dtype=info.dtype)])
        rng.shuffle(keys)
        grads = (rng.standard_normal((len(keys), DIM)) * 1e-2).astype(np.float32)
        k = torch.from_numpy(keys).cuda()
        out = torch.empty((len(keys), DIM), dtype=torch.float32, device="cuda")
        N.check(L.se_exchange_lookup(ex, k.data_ptr(), len(keys), out.data_ptr(), 1, C.c_void_p(st)))
        want = single.lookup_or_insert(keys, DIM)
        if step == 0:
            np.testing.assert_array_equal(out.cpu().numpy().ravel().view(np.uint32), want.view(np.uint32))
        else:
            np.testing.assert_allclose(out.cpu().numpy().ravel(), want, rtol=1e-5, atol=5e-7)
        g = torch.from_numpy(grads).cuda()
        if step == 3:
            N.check(L.se_exchange_accumulate(ex, k.data_ptr(), len(keys), g.data_ptr(), C.c_void_p(st)))
        else:
            N.check(L.se_exchange_accumulate_routed(ex, g.data_ptr(), len(keys), C.c_void_p(st)))
        single.accumulate_gradients(keys, grads, DIM)
        store.optimizer_step(1)
        single.optimizer_step(1)
        N.check(L.se_exchange_check(ex, C.c_void_p(st)))
    pk = torch.from_numpy(pool).cuda()
    out = torch.empty((len(pool), DIM), dtype=torch.float32, device="cuda")
    N.check(L.se_exchange_lookup(ex, pk.data_ptr(), len(pool), out.data_ptr(), 0, C.c_void_p(st)))
    np.testing.assert_allclose(out.cpu().numpy().ravel(), single.lookup(pool, DIM), rtol=1e-5, atol=5e-7)
    assert store.total_size() == single.size()
    N.check(L.se_exchange_check(ex, C.c_void_p(st)))
    N.check(L.se_exchange_destroy(ex))


def test_exchange_rejects_batches_above_its_capacity():
    L = N.lib()
    store = _store()
    ex = _exchange(store, 1, 0, 128)
    _connect_local([ex])
    k = torch.zeros(129, dtype=torch.int64, device="cuda")
    out = torch.empty((129, DIM), dtype=torch.float32, device="cuda")
    g = torch.zeros((129, DIM), dtype=torch.float32, device="cuda")
    rc = L.se_exchange_accumulate_routed(ex, g.data_ptr(), 129, None)
    assert rc == N.SE_ERR_INVALID_ARGUMENT
    assert b"no lookup" in L.se_last_error()
    rc = L.se_exchange_lookup(ex, k.data_ptr(), 129, out.data_ptr(), 1, None)
    assert rc == N.SE_ERR_INVALID_ARGUMENT
    assert b"max_keys_per_rank" in L.se_last_error()
    N.check(L.se_exchange_lookup(ex, k.data_ptr(), 100, out.data_ptr(), 1, None))
    rc = L.se_exchange_accumulate_routed(ex, g.data_ptr(), 99, None)
    assert rc == N.SE_ERR_INVALID_ARGUMENT
    assert b"must match the keys of the last lookup" in L.se_last_error()
    N.check(L.se_exchange_check(ex, None))
    N.check(L.se_exchange_destroy(ex))


def test_exchange_wait_gives_up_when_a_rank_is_absent():
    L = N.lib()
    torch.cuda.set_device(0)
    store = _store()
    ends = [_exchange(store, 2, r, 1024, timeout_ms=300) for r in range(2)]
    _connect_local(ends)
    st = torch.cuda.current_stream().cuda_stream
    k = torch.arange(100, dtype=torch.int64, device="cuda")
    out = torch.empty((100, DIM), dtype=torch.float32, device="cuda")
    # only rank 0 takes part: rank 1 never raises its flags
    N.check(L.se_exchange_lookup(ends[0], k.data_ptr(), 100, out.data_ptr(), 1, C.c_void_p(st)))
    rc = L.se_exchange_check(ends[0], C.c_void_p(st))
    assert rc == N.SE_ERR_RUNTIME
    assert b"timed out" in L.se_last_error()
    # the context is still usable
    rows, _ = store.lookup_or_insert(k, DIM)
    torch.cuda.synchronize()
    assert rows.numel() == 100 * DIM
    for h in ends:
        N.check(L.se_exchange_destroy(h))
