"""PyTorch autograd wrapper of the store's embedding bag: the forward is
EmbeddingStore.embedding_bag, the backward accumulates the pooled gradients
into the store (EmbeddingStore.embedding_bag_backward); the parameters are
updated by EmbeddingStore.optimizer_step, outside autograd.
"""

from __future__ import annotations

import torch


class EmbeddingBagFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, store, keys, offsets, dim, insert):
        ctx.store, ctx.keys, ctx.offsets = store, keys, offsets
        return store.embedding_bag(keys, offsets, dim, insert=insert)

    @staticmethod
    def backward(ctx, grad):
        ctx.store.embedding_bag_backward(ctx.keys, ctx.offsets, grad.contiguous())
        return None, None, None, None, None, None


def embedding_bag(store, keys: torch.Tensor, offsets: torch.Tensor, dim: int, insert: bool = True) -> torch.Tensor:
    """Sum-pooled bag rows [num_bags, dim] that take part in autograd: calling
    backward on a loss built from them accumulates the bags' gradients into
    `store` for its next optimizer_step."""
    anchor = torch.empty(0, device=keys.device, requires_grad=True)
    return EmbeddingBagFunction.apply(anchor, store, keys, offsets, dim, insert)
