"""ep.py — expert parallelism over the GPUs of one node, the host side.

Routed experts shard by expert id: rank r of n owns the experts e with
e % n == r, round-robin, so neighbouring ids (and the hot experts of a
skewed load, which land on ids at random) spread over the ranks.  Every
rank holds the layer's router, codebooks and shared expert, routes all T
tokens of a step identically, and runs only its own experts
(warp_moe_layer_forward_ep).  Those write slots [T][K + 1][hidden]:

* slot (t, j < K): route j's unweighted output if this rank owns its expert,
  else 0;
* slot (t, K): the shared expert's output for the tokens
  shared_tokens(T, r, n) of this rank, else 0.

One all-reduce (sum) over the ranks then hands every rank every slot.
Each slot has exactly one non-zero contributor, so the sum is exact in
any order. warp_moe_layer_combine finishes the layer on each rank in the
single-GPU order. The result is the one-GPU layer's, bit for bit.

The reference runs the experts of a token inside one process and sums them
in route order (model.c:4182-4241, 5858-5869); this keeps that reduction
and spreads the expert loop over GPUs.
"""
import torch


def owned_experts(n_experts, rank, size):
    """Expert ids rank `rank` of `size` holds, in the order of its bank."""
    if not 0 <= rank < size <= n_experts:
        raise ValueError("need 0 <= rank < size <= n_experts")
    return list(range(rank, n_experts, size))


def owner(expert, size):
    """The rank holding `expert`."""
    return expert % size


def shared_tokens(T, rank, size):
    """[t0, t1): the tokens whose shared expert rank `rank` computes."""
    return T * rank // size, T * (rank + 1) // size


def slot_shape(T, top_k, hidden):
    return (T, top_k + 1, hidden)


def all_reduce_slots(slots, group=None):
    """Sum the slots over the ranks (a no-op on one process)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(slots, op=dist.ReduceOp.SUM, group=group)
    return slots


class EPLayer:
    """One expert-parallel MoE layer on this rank: forward_ep, the slot
    all-reduce, combine.  `moe` is an ops.MoELayer created with this rank's
    bank and ep_rank/ep_size (or any object with the same three methods)."""

    def __init__(self, moe, group=None):
        self.moe = moe
        self.group = group
        self.slots = None

    def _slots(self, T, device):
        if self.slots is None or self.slots.shape[0] != T:
            self.slots = self.moe.slots(T, device)
        return self.slots

    def forward(self, x, residual=None, out=None):
        T = x.reshape(-1, self.moe.hidden).shape[0]
        slots = self._slots(T, x.device)
        self.moe.forward_ep(x, slots)
        all_reduce_slots(slots, self.group)
        return self.moe.combine(slots, residual, out)

