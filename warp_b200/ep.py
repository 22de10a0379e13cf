"""ep.py — expert parallelism over the GPUs of one node, the host side.

Two ways to split a layer's routed experts over n ranks (warp_moe_desc
ep_mode):

* mode 0, by expert id: rank r holds the experts e with e % n == r,
  round-robin (neighbouring ids, and the hot experts of a skewed load,
  which land on ids at random, spread over the ranks), and computes the
  routes that pick them.  Each rank's bank holds 1/n of the experts: the
  split that lets a model larger than one GPU stay resident.
* mode 1, routes dealt: every rank holds all experts (the layer fits one
  GPU) and rank r computes the routes t*K + j with (t*K + j) % n == r,
  which balances the ranks exactly whatever the routing skew.

Every rank holds the layer's router, codebooks and shared expert and routes
all T tokens of a step identically.  The shared expert's down projection is
computed in nb fixed column blocks (shared_blocks); rank r computes blocks
[nb*r/n, nb*(r+1)/n) and the gate/up rows that feed them.
warp_moe_layer_forward_ep writes slots [T][K + nb][hidden]:

* slot (t, j < K): route j's unweighted output if this rank computes it,
  else 0;
* slot (t, K + b): the shared expert's partial over column block b if this
  rank computes it, else 0.

One all-reduce (sum) over the ranks then hands every rank every slot.
Each slot has exactly one non-zero contributor, so the sum is exact in
any order. warp_moe_layer_combine finishes the layer on each rank in the
single-GPU order (routes in route order, then the nb partials in block
order). The result is the one-GPU layer's, bit for bit.

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


def route_owner(route, size):
    """Mode 1: the rank computing route t*K + j."""
    return route % size


def shared_blocks(shared_inter, group):
    """nb, the shared expert's column blocks: 8, 4, 2 or 1, the largest whose
    blocks are whole groups (the rule warp_moe_layer_create applies)."""
    for nb in (8, 4, 2, 1):
        if shared_inter % (nb * group) == 0:
            return nb
    return 1


def shared_block_span(nb, rank, size):
    """[b0, b1): the shared-expert column blocks rank `rank` computes."""
    return nb * rank // size, nb * (rank + 1) // size


def slot_shape(T, top_k, hidden, nb):
    return (T, top_k + nb, hidden)


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

