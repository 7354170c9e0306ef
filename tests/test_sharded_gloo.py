"""Exchange bookkeeping of ShardedEmbeddingStore on CPU ranks (gloo, world 2).

The routing and the local stores are CPU stand-ins built on the oracle (test
infrastructure); the all-to-all plan, splits, row return order and gradient
routing are the production code. Results must equal one oracle store fed the
concatenation of the ranks' batches, bit for bit.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

DIM = 16
WORLD = 2


class OracleRouter:
    def __init__(self, kind, world):
        self.kind, self.world = kind, world

    def route(self, keys):
        from oracle import oracle as O

        k = keys.numpy()
        ids = O.partition(self.kind, self.world, k)
        order = np.argsort(ids, kind="stable")
        counts = np.bincount(ids, minlength=self.world).astype(np.int32)
        return (torch.from_numpy(k[order].copy()), torch.from_numpy(order.astype(np.int32)),
                torch.from_numpy(counts))

    def to_routed(self, rows, positions):
        return rows[positions.long()]

    def from_routed(self, rows, positions):
        out = torch.empty_like(rows)
        out[positions.long()] = rows
        return out


class OracleLocal:
    """Local store stand-in with the EmbeddingStore call shapes, on CPU tensors."""

    def __init__(self, ref):
        self.ref = ref

    def lookup_or_insert(self, keys, dim):
        return torch.from_numpy(self.ref.lookup_or_insert(keys.numpy(), dim)), None

    def lookup(self, keys, dim):
        return torch.from_numpy(self.ref.lookup(keys.numpy(), dim)), None

    def accumulate_gradients(self, keys, grads):
        self.ref.accumulate_gradients(keys.numpy(), grads.numpy(), DIM)

    def optimizer_step(self, n):
        self.ref.optimizer_step(n)


def batches(rank, steps, rng_seed=0):
    rng = np.random.default_rng([rng_seed, rank])
    pool = np.random.default_rng(99).integers(-2**63, 2**63 - 1, size=300, dtype=np.int64)
    out = []
    for _ in range(steps):
        keys = np.concatenate([rng.choice(pool, size=500), rng.integers(-2**63, 2**63 - 1, size=20, dtype=np.int64)])
        grads = (rng.standard_normal((len(keys), DIM)) * 1e-2).astype(np.float32)
        out.append((keys, grads))
    return out, pool


def _worker(rank, port, kind, steps, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from oracle import oracle as O
        from sparse_embedding_b200.sharded import ShardedEmbeddingStore

        local = OracleLocal(O.OracleStore([DIM], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8,
                                          initial_accumulator=0.1))
        sharded = ShardedEmbeddingStore(local, router=OracleRouter(kind, WORLD))
        mine, pool = batches(rank, steps)
        rows_seen = []
        for keys, grads in mine:
            k = torch.from_numpy(keys)
            rows = sharded.lookup_or_insert(k, DIM)
            rows_seen.append(rows.numpy().copy())
            sharded.accumulate_gradients(k, torch.from_numpy(grads))
            sharded.optimizer_step(1)
        final = sharded.lookup(torch.from_numpy(pool), DIM).numpy()
        q.put((rank, rows_seen, final))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("kind", ["hash", "modulo"])
def test_sharded_exchange_matches_single_store(kind):
    from oracle import oracle as O

    steps = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, kind, steps, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict((r, (rows, final)) for r, rows, final in (q.get(timeout=120) for _ in range(WORLD)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    # One store fed the concatenated global batch of every step.
    single = O.OracleStore([DIM], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8, initial_accumulator=0.1)
    per_rank = [batches(r, steps)[0] for r in range(WORLD)]
    pool = batches(0, steps)[1]
    for s in range(steps):
        for r in range(WORLD):
            keys, _ = per_rank[r][s]
            want = single.lookup_or_insert(keys, DIM)
            np.testing.assert_array_equal(results[r][0][s].ravel().view(np.uint32), want.view(np.uint32))
        for r in range(WORLD):
            keys, grads = per_rank[r][s]
            single.accumulate_gradients(keys, grads, DIM)
        single.optimizer_step(1)
    want = single.lookup(pool, DIM)
    for r in range(WORLD):
        np.testing.assert_array_equal(results[r][1].ravel().view(np.uint32), want.view(np.uint32))
