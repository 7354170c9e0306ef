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
