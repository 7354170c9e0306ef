"""Train steps captured as CUDA graphs (as bench.py times them) produce the
same table as the same calls made eagerly (GPU)."""

import numpy as np
import pytest
import torch

import sparse_embedding_b200 as se
from sparse_embedding_b200.workloads import TrainWorkload

pytestmark = pytest.mark.gpu


def _store(cap):
    return se.EmbeddingStore(se.EmbeddingConfig(dims=[64], key_dtype="int64", initial_capacity=cap),
                             optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))


def test_graph_replay_matches_eager():
    wl = TrainWorkload(num_keys=50_000, batch=8192)
    keys_np, grads_np = wl.make_batches(8)
    keys = torch.from_numpy(keys_np).cuda()
    grads = torch.from_numpy(grads_np).cuda()
    warm = torch.from_numpy(wl.warm_keys()).cuda()
    eager, graphed = _store(200_000), _store(200_000)
    for st in (eager, graphed):
        st.lookup_or_insert(warm, 64)

    def step(st, s):
        k = keys[s]
        st.lookup_or_insert(k, 64)
        st.accumulate_gradients(k, grads[s])
        st.optimizer_step(1)

    for s in range(8):
        step(eager, s)
    for s in range(3):  # warm-up sizes the work buffers before capture
        step(graphed, s)
    pool = torch.cuda.graph_pool_handle()
    graphs = []
    for s in range(3, 8):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool, capture_error_mode="relaxed"):
            step(graphed, s)
        graphs.append(g)
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    probe = torch.unique(torch.cat([keys.flatten(), warm[:1000]]))
    a, _ = eager.lookup(probe, 64)
    b, _ = graphed.lookup(probe, 64)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    assert eager.total_size() == graphed.total_size()


def test_insert_captured_after_eager_calls_finds_room():
    """The table's row bound carries every insert call's whole batch (new
    rows are known only on the device). After eager calls that bring the
    bound near the capacity, a call of the same size captured next in a CUDA
    graph - which can neither read the rows in use nor grow the arena - still
    finds its room: every uncaptured call leaves room for one more of its
    size, reading the rows in use again when the bound leaves less."""
    n, used = 65_536, 100_000
    cap = used + 5 * n // 2
    st = se.EmbeddingStore(se.EmbeddingConfig(dims=[16], key_dtype="int64", initial_capacity=cap),
                           optimizer_config=se.Sgd(lr=0.01))
    keys = torch.arange(1, used + 1, dtype=torch.int64, device="cuda")
    st.lookup_or_insert(keys, 16)
    batch = keys[:n].clone()
    for _ in range(2):
        st.lookup_or_insert(batch, 16)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rows, _ = st.lookup_or_insert(batch, 16)
    g.replay()
    torch.cuda.synchronize()
    want, _ = st.lookup(batch, 16)
    assert torch.equal(rows.view(torch.int32), want.view(torch.int32))
    assert st.total_size() == used
    del g
