"""Key-sharded store on 2 GPUs against one oracle store fed the concatenated
global batches (GPU, needs 2 devices), over both transports: NCCL
all-to-all ("collective") and the library's peer-memory exchange ("p2p")."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.test_sharded_gloo import DIM, batches

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, kind, transport, steps, q, accumulation="ordered", dedupe=False):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import sparse_embedding_b200 as se
        from sparse_embedding_b200.sharded import ShardedEmbeddingStore

        store = se.EmbeddingStore(se.EmbeddingConfig(dims=[DIM], key_dtype="int64", device=rank,
                                                     accumulation=accumulation),
                                  optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))
        sharded = ShardedEmbeddingStore(store, f"sparse_embedding.{kind}", transport=transport,
                                        max_keys_per_rank=1024, timeout_ms=20_000, dedupe=dedupe)
        mine, pool = batches(rank, steps)
        rows_seen = []
        for s, (keys, grads) in enumerate(mine):
            k = torch.from_numpy(keys).cuda()
            rows = sharded.lookup_or_insert(k, DIM)
            rows_seen.append(rows.cpu().numpy().copy())
            # odd steps pass a copy of the keys: the gradient batch is routed by its own keys
            sharded.accumulate_gradients(k if s % 2 == 0 else k.clone(), torch.from_numpy(grads).cuda())
            sharded.optimizer_step(1)
        final = sharded.lookup(torch.from_numpy(pool).cuda(), DIM).cpu().numpy()
        sharded.check()
        torch.cuda.synchronize()
        sharded.close()
        q.put((rank, rows_seen, final))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["collective", "p2p", "p2p-dedupe"])
@pytest.mark.parametrize("kind", ["hash", "fast_range"])
@pytest.mark.parametrize("accumulation", ["ordered", "atomic"])
def test_sharded_two_gpus_match_single_store(kind, transport, accumulation):
    """Ordered accumulation over the plain routes: bit for bit. Atomic
    accumulation (per-key fp32 sums, order of the adds varies) or sender-side
    dedupe (gradients pre-summed per key on the sender): the first step's
    rows bit for bit, the rest within 1e-5 relative (atol 1e-5 of the
    values' 0.05 scale)."""
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    from oracle import oracle as O

    steps = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    dedupe = transport == "p2p-dedupe"
    procs = [ctx.Process(target=_worker, args=(r, port, kind, "p2p" if dedupe else transport, steps, q,
                                               accumulation, dedupe))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict((r, (rows, final)) for r, rows, final in (q.get(timeout=300) for _ in range(WORLD)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    single = O.OracleStore([DIM], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8, initial_accumulator=0.1)
    per_rank = [batches(r, steps)[0] for r in range(WORLD)]
    pool = batches(0, steps)[1]
    exact = accumulation == "ordered" and not dedupe
    for s in range(steps):
        for r in range(WORLD):
            want = single.lookup_or_insert(per_rank[r][s][0], DIM)
            got = results[r][0][s].ravel()
            if exact or s == 0:
                np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
            else:
                np.testing.assert_allclose(got, want, rtol=1e-5, atol=5e-7)
        for r in range(WORLD):
            single.accumulate_gradients(per_rank[r][s][0], per_rank[r][s][1], DIM)
        single.optimizer_step(1)
    want = single.lookup(pool, DIM)
    for r in range(WORLD):
        if exact:
            np.testing.assert_array_equal(results[r][1].ravel().view(np.uint32), want.view(np.uint32))
        else:
            np.testing.assert_allclose(results[r][1].ravel(), want, rtol=1e-5, atol=5e-7)


def _mixed_batches(rank, steps):
    """int32 keys incl. negatives, a few keys with far more than 64 rows per
    step across the two ranks (the hot-key reduction), fp16 gradients."""
    rng = np.random.default_rng([7, rank])
    pool = np.random.default_rng(5).integers(-2**31, 2**31 - 1, size=400, dtype=np.int32)
    out = []
    for _ in range(steps):
        keys = np.concatenate([rng.choice(pool, size=700), np.repeat(pool[:3], 60),
                               rng.integers(-2**31, 2**31 - 1, size=30, dtype=np.int32)])
        rng.shuffle(keys)
        grads = (rng.standard_normal((len(keys), MIXED_DIM)) * 1e-2).astype(np.float16)
        out.append((keys, grads))
    return out, pool


MIXED_DIM = 24


def _worker_mixed(rank, port, steps, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import sparse_embedding_b200 as se
        from sparse_embedding_b200.sharded import ShardedEmbeddingStore

        store = se.EmbeddingStore(se.EmbeddingConfig(dims=[MIXED_DIM], key_dtype="int32", value_dtype="float16",
                                                     optimizer_dtype="float32", gradient_dtype="float16",
                                                     device=rank),
                                  optimizer_config=se.Adam(lr=1e-3))
        sharded = ShardedEmbeddingStore(store, "sparse_embedding.modulo", transport="p2p", max_keys_per_rank=1024,
                                        timeout_ms=20_000)
        mine, pool = _mixed_batches(rank, steps)
        rows_seen = []
        for keys, grads in mine:
            k = torch.from_numpy(keys).cuda()
            rows = sharded.lookup_or_insert(k, MIXED_DIM)
            rows_seen.append(rows.view(torch.int16).cpu().numpy().copy())
            sharded.accumulate_gradients(k, torch.from_numpy(grads).cuda())
            sharded.optimizer_step(1)
        final = sharded.lookup(torch.from_numpy(pool).cuda(), MIXED_DIM).float().cpu().numpy()
        sharded.check()
        torch.cuda.synchronize()
        sharded.close()
        q.put((rank, rows_seen, final))
    finally:
        dist.destroy_process_group()


def test_sharded_two_gpus_int32_fp16_adam_hot_keys_p2p():
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    from oracle import oracle as O

    steps = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_mixed, args=(r, port, steps, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict((r, (rows, final)) for r, rows, final in (q.get(timeout=300) for _ in range(WORLD)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    single = O.OracleStore([MIXED_DIM], key_dtype="int32", value_dtype="float16", optimizer_dtype="float32",
                           gradient_dtype="float16", optimizer="adam", lr=1e-3)
    per_rank = [_mixed_batches(r, steps)[0] for r in range(WORLD)]
    pool = _mixed_batches(0, steps)[1]
    for s in range(steps):
        for r in range(WORLD):
            want = single.lookup_or_insert(per_rank[r][s][0], MIXED_DIM)
            got = results[r][0][s].ravel().view(np.uint16)
            if s == 0:
                np.testing.assert_array_equal(got, want)
            else:  # fp16 parameters: within one fp16 ulp of the oracle (hot keys reduced in parallel runs)
                np.testing.assert_allclose(got.view(np.float16).astype(np.float32),
                                           want.view(np.float16).astype(np.float32), rtol=1e-3, atol=1e-5)
        for r in range(WORLD):
            single.accumulate_gradients(per_rank[r][s][0], per_rank[r][s][1].view(np.uint16), MIXED_DIM)
        single.optimizer_step(1)
    want = single.lookup(pool, MIXED_DIM).view(np.float16).astype(np.float32)
    for r in range(WORLD):
        np.testing.assert_allclose(results[r][1].ravel(), want, rtol=1e-3, atol=1e-5)
