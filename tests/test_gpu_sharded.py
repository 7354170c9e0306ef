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


def _worker(rank, port, kind, transport, steps, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import sparse_embedding_b200 as se
        from sparse_embedding_b200.sharded import ShardedEmbeddingStore

        store = se.EmbeddingStore(se.EmbeddingConfig(dims=[DIM], key_dtype="int64", device=rank),
                                  optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))
        sharded = ShardedEmbeddingStore(store, f"sparse_embedding.{kind}", transport=transport,
                                        max_keys_per_rank=1024, timeout_ms=20_000)
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


@pytest.mark.parametrize("transport", ["collective", "p2p"])
@pytest.mark.parametrize("kind", ["hash", "fast_range"])
def test_sharded_two_gpus_match_single_store(kind, transport):
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    from oracle import oracle as O

    steps = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, kind, transport, steps, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict((r, (rows, final)) for r, rows, final in (q.get(timeout=300) for _ in range(WORLD)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    single = O.OracleStore([DIM], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8, initial_accumulator=0.1)
    per_rank = [batches(r, steps)[0] for r in range(WORLD)]
    pool = batches(0, steps)[1]
    for s in range(steps):
        for r in range(WORLD):
            want = single.lookup_or_insert(per_rank[r][s][0], DIM)
            np.testing.assert_array_equal(results[r][0][s].ravel().view(np.uint32), want.view(np.uint32))
        for r in range(WORLD):
            single.accumulate_gradients(per_rank[r][s][0], per_rank[r][s][1], DIM)
        single.optimizer_step(1)
    want = single.lookup(pool, DIM)
    for r in range(WORLD):
        np.testing.assert_array_equal(results[r][1].ravel().view(np.uint32), want.view(np.uint32))
