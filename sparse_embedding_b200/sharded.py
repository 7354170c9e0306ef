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

The collectives are torch.distributed all_to_all_single calls (NCCL on GPUs).
The routing and permutation steps are sm_100a kernels by default
(GpuRouter); any object with the same three methods can stand in for it.
"""

from __future__ import annotations

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


class ShardedEmbeddingStore:
    """Data-parallel batches over key-sharded stores, one per rank."""

    def __init__(self, local_store, partitioner_name: str = "sparse_embedding.hash", group=None, router=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.store = local_store
        self.router = router if router is not None else GpuRouter(partitioner_name, self.world)
        self._plan: ExchangePlan | None = None
        self._plan_keys = None

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
        plan = self._plan_for(keys)
        dim = grads.shape[-1]
        routed = self.router.to_routed(grads.reshape(-1, dim), plan.send_positions)
        recv = routed.new_empty((sum(plan.recv_splits), dim))
        self.dist.all_to_all_single(recv, routed, plan.recv_splits, plan.send_splits, group=self.group)
        self.store.accumulate_gradients(plan.recv_keys, recv)

    def optimizer_step(self, normalization_steps: int) -> None:
        self.store.optimizer_step(normalization_steps)
