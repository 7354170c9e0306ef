"""se_partition_route_noalloc against se_partition_route, through the C ABI (GPU).

The no-allocation variant exists for callers that cannot allocate device
memory during a step (a host framework whose allocator already holds the
device's memory, or a serving loop that must not fail or stall on an
allocation mid-batch). Its scratch is one fixed array shared by every call,
so this test makes two calls in a row with different inputs and checks both
against the allocating entry point; the outputs are integers and must match
exactly. The file is named to be collected last.
"""

import numpy as np
import pytest
import torch

from sparse_embedding_b200 import _native as N

pytestmark = pytest.mark.gpu


def _route(fn, kind, parts, keys):
    n = keys.numel()
    send_keys = torch.empty_like(keys)
    send_pos = torch.empty(n, dtype=torch.int32, device=keys.device)
    counts = torch.empty(parts, dtype=torch.int32, device=keys.device)
    st = torch.cuda.current_stream().cuda_stream
    N.check(fn(kind, parts, N.KEY_CODES[str(keys.dtype).replace("torch.", "")], keys.data_ptr(), n,
               send_keys.data_ptr(), send_pos.data_ptr(), counts.data_ptr(), keys.device.index, st))
    torch.cuda.synchronize()
    return send_keys.cpu(), send_pos.cpu(), counts.cpu()


def test_noalloc_route_matches_allocating_route_twice():
    L = N.lib()
    torch.cuda.set_device(0)
    cases = [  # (kind, partitions, keys): two calls in a row, different shapes and dtypes
        (N.PART_CODES["hash"], 8, torch.randint(-2**62, 2**62, (300_001,), dtype=torch.int64, device="cuda")),
        (N.PART_CODES["modulo"], 3, torch.randint(0, 2**31 - 1, (77_777,), dtype=torch.int32, device="cuda")),
    ]
    for kind, parts, keys in cases:
        want = _route(L.se_partition_route, kind, parts, keys)
        got = _route(L.se_partition_route_noalloc, kind, parts, keys)
        for w, g in zip(want, got):
            assert torch.equal(w, g)
        assert int(got[2].sum()) == keys.numel()


def test_noalloc_route_rejects_inputs_beyond_its_scratch():
    L = N.lib()
    keys = torch.zeros(2048 * 8193, dtype=torch.int64, device="cuda")  # 8193 tiles x 8 partitions > 65536
    out = torch.empty_like(keys)
    pos = torch.empty(keys.numel(), dtype=torch.int32, device="cuda")
    counts = torch.empty(8, dtype=torch.int32, device="cuda")
    rc = L.se_partition_route_noalloc(N.PART_CODES["hash"], 8, N.KEY_CODES["int64"], keys.data_ptr(), keys.numel(),
                                      out.data_ptr(), pos.data_ptr(), counts.data_ptr(), 0,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == N.SE_ERR_INVALID_ARGUMENT
    assert b"exceeds its fixed scratch" in L.se_last_error()
