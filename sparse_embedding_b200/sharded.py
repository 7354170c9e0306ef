"""Key-sharded store over several GPUs (one process per GPU).

The reference leaves cross-worker routing to its caller
(sparse_embedding/partitioner.py:84-100, a FunctionPartition contract); this
module is that caller for N GPUs: rank r owns the keys the configured
partitioner maps to r, and every data-parallel batch is exchanged once each
way:

  forward : route keys by owner (stable) -> all-to-all counts -> all-to-all
            keys -> owner lookup_or_insert -> all-to-all rows back -> rows
            restored to the batch order;
  backward: gradient rows permuted to the routed order -> all-to-all ->
            owner accumulate_gradients;
  step    : each owner applies its optimizer locally (no all-reduce).

Ownership is a pure function of the key, so the rows and optimizer state a
key reaches do not depend on the number of GPUs; received batches are laid
out rank 0 first, so an owner accumulates a key's gradients in the order of
the concatenated global batch.

Two transports carry the exchange:

  "collective": torch.distributed all_to_all_single calls (NCCL on GPUs, gloo
                on CPU). The routing and permutation steps are sm_100a kernels
                by default (GpuRouter); any object with the same three methods
                can stand in for it.
  "p2p"       : the library's peer-memory exchange (se_exchange_*): every rank
                maps every rank's exchange arena through CUDA IPC and the
                route, scatter, owner lookup / insert and row return are
                kernels that store straight into the peers' HBM over NVLink,
                synchronised by flags in device memory - no host round trip,
                no collective library, and capturable in a CUDA graph.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _native as N
from ._tensors import torch_mod
from .partitioner import create_partitioner


class GpuRouter:
    """Routing and row permutation kernels of libse_gpu.so."""

    def __init__(self, partitioner_name: str, world: int):
        self.part = create_partitioner(partitioner_name, world)

    def route(self, keys):
        """(send_keys, send_positions int32, counts int32[world]) grouped by owner, stable."""
        return self.part.route(keys)

    def to_routed(self, rows, positions):
        """out[j] = rows[positions[j]]"""
        return self._permute(rows, positions, scatter=1)

    def from_routed(self, rows, positions):
        """out[positions[j]] = rows[j]"""
        return self._permute(rows, positions, scatter=0)

    @staticmethod
    def _permute(rows, positions, scatter: int):
        torch = torch_mod()
        out = torch.empty_like(rows)
        n = rows.shape[0]
        if n:
            row_bytes = rows.element_size() * (rows.numel() // n)
            st = torch.cuda.current_stream(rows.device).cuda_stream
            N.check(N.lib().se_permute_rows(rows.data_ptr(), out.data_ptr(), positions.data_ptr(), n, row_bytes,
                                            scatter, rows.device.index, st))
        return out


@dataclass
class ExchangePlan:
    send_positions: object
    send_splits: list
    recv_splits: list
    recv_keys: object


class PeerExchange:
    """One rank's end of the peer-memory exchange for rows of length `dim`.

    Collective: every rank of `group` constructs it with the same arguments
    and then makes the same sequence of lookup / accumulate calls. Without an
    initialised process group it is a one-rank exchange (every key owned
    locally), which runs the same kernels on one GPU.
    """

    HANDLE_BYTES = 64  # a CUDA IPC memory handle

    def __init__(self, store, partitioner_name: str, dim: int, max_keys_per_rank: int, group=None,
                 timeout_ms: int = 10_000, dedupe: bool = False):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.store = store
        self.dim = int(dim)
        self.max_keys = int(max_keys_per_rank)
        self._lib = N.lib()
        self._last_keys = None  # keys tensor of the last lookup
        kind = create_partitioner(partitioner_name, self.world)._kind
        h = C.c_void_p()
        N.check(self._lib.se_exchange_create(store._h, N.PART_CODES[kind], self.world, self.rank, self.max_keys,
                                             self.dim, int(timeout_ms), C.byref(h)))
        self._h = h
        # every distinct key of a batch is routed once; the routed gradients
        # are summed per key on the sender (fp32) before they are sent
        N.check(self._lib.se_exchange_set_dedupe(h, int(bool(dedupe))))
        if not self.distributed:
            N.check(self._lib.se_exchange_connect_local((C.c_void_p * 1)(h.value), 1))
            return
        buf = (C.c_char * self.HANDLE_BYTES)()
        N.check(self._lib.se_exchange_handle(h, buf, self.HANDLE_BYTES))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(buf), group=group)
        joined = b"".join(handles)
        N.check(self._lib.se_exchange_connect(h, joined, len(joined)))
        dist.barrier(group)  # every arena is mapped before any rank stores into it

    def _stream(self, t):
        torch = torch_mod()
        return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)

    def lookup(self, keys, insert: bool, out=None):
        """(n, dim) rows of this rank's keys in batch order, from their owners."""
        torch = torch_mod()
        n = keys.numel()
        if out is None:
            out = torch.empty((n, self.dim), dtype=getattr(torch, self.store.value_dtype()), device=keys.device)
        N.check(self._lib.se_exchange_lookup(self._h, keys.data_ptr(), n, out.data_ptr(), int(insert),
                                             self._stream(keys)))
        self._last_keys = keys
        return out

    def accumulate(self, keys, grads) -> None:
        """Sends grads[i] (gradient dtype, (n, dim)) of keys[i] to the key's owner.

        When `keys` is the tensor of the last lookup (the usual forward ->
        backward pair), the rows follow that lookup's route and no keys are
        sent again; like the collective transport's plan cache, this assumes
        the tensor was not modified in between.
        """
        if keys is self._last_keys:
            N.check(self._lib.se_exchange_accumulate_routed(self._h, grads.data_ptr(), keys.numel(),
                                                            self._stream(keys)))
            return
        N.check(self._lib.se_exchange_accumulate(self._h, keys.data_ptr(), keys.numel(), grads.data_ptr(),
                                                 self._stream(keys)))

    def check(self) -> None:
        """Waits for this rank's stream; raises a timed-out exchange or table errors."""
        torch = torch_mod()
        N.check(self._lib.se_exchange_check(self._h, C.c_void_p(torch.cuda.current_stream().cuda_stream)))

    def close(self) -> None:
        if self._h is not None:
            torch = torch_mod()
            torch.cuda.synchronize()
            if self.distributed:
                self.dist.barrier(self.group)  # no peer stores into this arena any more
            N.check(self._lib.se_exchange_destroy(self._h))
            self._h = None


class ShardedEmbeddingStore:
    """Data-parallel batches over key-sharded stores, one per rank."""

    def __init__(self, local_store, partitioner_name: str = "sparse_embedding.hash", group=None, router=None,
                 transport: str = "collective", max_keys_per_rank: int | None = None, timeout_ms: int = 10_000,
                 dedupe: bool = False):
        import torch.distributed as dist

        if transport not in ("collective", "p2p"):
            raise ValueError("transport must be 'collective' or 'p2p'")
        if transport == "p2p" and not max_keys_per_rank:
            raise ValueError("the p2p transport needs max_keys_per_rank")
        self.dist = dist
        self.group = group
        distributed = dist.is_available() and dist.is_initialized()
        if transport == "collective" and not distributed:
            raise ValueError("the collective transport needs an initialised process group")
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        self.store = local_store
        self.partitioner_name = partitioner_name
        self.transport = transport
        self.max_keys_per_rank = max_keys_per_rank
        self.timeout_ms = timeout_ms
        # p2p: route each distinct key of a batch once per sender and sum its
        # gradient rows on the sender (rows unchanged; updates within fp32
        # reassociation of the plain route)
        self.dedupe = bool(dedupe)
        self._exchanges: dict[int, PeerExchange] = {}
        self.router = router if router is not None else (
            GpuRouter(partitioner_name, self.world) if transport == "collective" else None)
        self._plan: ExchangePlan | None = None
        self._plan_keys = None

    def exchange(self, dim: int) -> PeerExchange:
        """The peer-memory exchange for rows of length dim (created on first use; collective)."""
        ex = self._exchanges.get(dim)
        if ex is None:
            ex = PeerExchange(self.store, self.partitioner_name, dim, self.max_keys_per_rank, self.group,
                              self.timeout_ms, dedupe=self.dedupe)
            self._exchanges[dim] = ex
        return ex

    def check(self) -> None:
        """p2p transport: waits for this rank's stream and raises exchange or table errors."""
        for ex in self._exchanges.values():
            ex.check()

    def close(self) -> None:
        """Releases the peer-memory exchanges (collective)."""
        for ex in self._exchanges.values():
            ex.close()
        self._exchanges.clear()

    # ---- exchange ------------------------------------------------------------

    def plan(self, keys) -> ExchangePlan:
        torch = torch_mod()
        send_keys, send_pos, counts = self.router.route(keys)
        recv_counts = torch.empty_like(counts)
        self.dist.all_to_all_single(recv_counts, counts, group=self.group)
        both = torch.stack([counts, recv_counts]).cpu()
        send_splits = [int(x) for x in both[0]]
        recv_splits = [int(x) for x in both[1]]
        recv_keys = send_keys.new_empty(sum(recv_splits))
        self.dist.all_to_all_single(recv_keys, send_keys, recv_splits, send_splits, group=self.group)
        plan = ExchangePlan(send_pos, send_splits, recv_splits, recv_keys)
        self._plan, self._plan_keys = plan, keys
        return plan

    def _plan_for(self, keys) -> ExchangePlan:
        if self._plan is not None and self._plan_keys is keys:
            return self._plan
        return self.plan(keys)

    # ---- hot path ------------------------------------------------------------

    def _rows(self, keys, dim: int, insert: bool):
        if self.transport == "p2p":
            return self.exchange(dim).lookup(keys, insert)
        plan = self.plan(keys)
        fn = self.store.lookup_or_insert if insert else self.store.lookup
        owned, _ = fn(plan.recv_keys, dim)
        owned = owned.view(-1, dim)
        back = owned.new_empty((sum(plan.send_splits), dim))
        self.dist.all_to_all_single(back, owned, plan.send_splits, plan.recv_splits, group=self.group)
        return self.router.from_routed(back, plan.send_positions)

    def lookup(self, keys, dim: int):
        """Rows of the batch's keys, in batch order (zeros for absent keys)."""
        return self._rows(keys, dim, insert=False)

    def lookup_or_insert(self, keys, dim: int):
        return self._rows(keys, dim, insert=True)

    def accumulate_gradients(self, keys, grads) -> None:
        """grads[i] is the gradient row of keys[i]; it is sent to the key's owner."""
        dim = grads.shape[-1]
        if self.transport == "p2p":
            self.exchange(dim).accumulate(keys, grads.reshape(-1, dim).contiguous())
            return
        plan = self._plan_for(keys)
        routed = self.router.to_routed(grads.reshape(-1, dim), plan.send_positions)
        recv = routed.new_empty((sum(plan.recv_splits), dim))
        self.dist.all_to_all_single(recv, routed, plan.recv_splits, plan.send_splits, group=self.group)
        self.store.accumulate_gradients(plan.recv_keys, recv)

    def optimizer_step(self, normalization_steps: int) -> None:
        self.store.optimizer_step(normalization_steps)
