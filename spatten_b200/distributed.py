"""Sharding over ranks (one process per GPU) and the importance all-reduces.

The (batch, head) units of the attention kernel are independent, so work is
partitioned without a collective on the data path. Two decisions of the
cascade are not local, and each needs exactly one all-reduce:

* Head pruning is batch-global in the reference: head importance is
  ``context.abs().mean(dim=(0, 2, 3))`` over the whole batch
  (spatten_bert.py:120-121). With the batch sharded, every rank all-reduces
  its per-head sums of |context| and the element count, so that all ranks
  take the same top-k and keep the same heads (``allreduce_head_importance``).
* Token importance sums over heads (spatten_bert.py:136). With heads split
  across ranks, every rank all-reduces its partial [B, S] sums before the
  token top-k (``allreduce_token_importance``).

Collectives go through ``torch.distributed`` (NCCL over NVLink on GPUs, gloo
on the CPU for tests) on the current stream.
"""
import torch
import torch.distributed as dist


def world():
    """(rank, world_size) of the default group, (0, 1) without one."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def shard_range(n, rank, world_size):
    """Contiguous [start, stop) of ``n`` units for ``rank`` (sizes differ by <= 1)."""
    base, extra = divmod(n, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(x, rank=None, world_size=None, dim=0):
    """This rank's slice of ``x`` along ``dim`` (the batch)."""
    if rank is None or world_size is None:
        rank, world_size = world()
    a, b = shard_range(x.shape[dim], rank, world_size)
    return x.narrow(dim, a, b - a)


def allreduce_head_importance(head_abs_sum, count, group=None):
    """Global mean |context| per head from per-rank sums.

    ``head_abs_sum`` [H] fp32: this rank's sum of |context| per head;
    ``count``: this rank's number of summed elements per head (B_local*S*D).
    Returns the batch-global mean, identical on every rank."""
    # built on the device (a host-made tensor would copy from pageable memory
    # and stall the host once per layer)
    n = head_abs_sum.numel()
    buf = torch.empty(n + 1, dtype=torch.float64, device=head_abs_sum.device)
    buf[:n].copy_(head_abs_sum.reshape(-1))
    buf[n:].fill_(float(count))
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    return (buf[:-1] / buf[-1]).to(torch.float32)


def allreduce_token_importance(tok, group=None):
    """Sum the per-rank partial token importance [B, S] (heads split across ranks)."""
    dist.all_reduce(tok, op=dist.ReduceOp.SUM, group=group)
    return tok


class HeadBatchShards:
    """Partition of a [B, H] grid of (batch, head) units over ``world`` ranks:
    the heads are split over ``head_ranks`` ranks (the largest divisor of H
    that divides ``world`` and is at most ``max_head_ranks``), the batch over
    the remaining ``world // head_ranks``. Rank r holds heads
    [h0, h1) of batch rows [b0, b1); the ranks that share its batch rows form
    its head group, over which the token importance is all-reduced.
    ``groups()`` must be called on every rank (it creates the process groups
    in the same order everywhere)."""

    def __init__(self, B, H, rank, world_size, max_head_ranks=4):
        hr = 1
        for c in range(1, min(max_head_ranks, world_size) + 1):
            if H % c == 0 and world_size % c == 0:
                hr = c
        br = world_size // hr
        if B % br:
            raise ValueError(f"batch {B} does not split over {br} ranks")
        self.B, self.H, self.rank, self.world = B, H, rank, world_size
        self.head_ranks, self.batch_ranks = hr, br
        hi, bi = rank % hr, rank // hr
        self.h0, self.h1 = hi * H // hr, (hi + 1) * H // hr
        self.b0, self.b1 = bi * B // br, (bi + 1) * B // br
        self._group = None

    def groups(self):
        """This rank's head group (None with one head rank)."""
        if self.head_ranks == 1:
            return None
        if self._group is None:
            mine = None
            for bi in range(self.batch_ranks):
                g = dist.new_group([bi * self.head_ranks + i for i in range(self.head_ranks)])
                if bi == self.rank // self.head_ranks:
                    mine = g
            self._group = mine
        return self._group

    def take(self, x):
        """This rank's units of a [B, H, ...] tensor."""
        return x[self.b0:self.b1, self.h0:self.h1]


def topk_by_batch_shard(importance, k, group=None, topk=None):
    """Token top-k of a summed importance [B, N] whose per-rank partial sums
    each rank holds (KV heads split over ranks), with the selection itself
    split over the batch: a reduce-scatter leaves each rank the summed rows
    of its B / world batch rows, the rank takes their top-k, and an
    all-gather of the kept indices gives every rank all B rows. Moves
    (world - 1) / world of the importance once instead of twice, and each
    rank selects B / world rows instead of B. B must be a multiple of the
    group size. ``topk(x, k)`` -> int64 [rows, k] ascending indices (the
    CUDA top-k by default). Returns (kept int64 [B, k], this rank's summed
    importance rows [B / world, N])."""
    if topk is None:
        from .select import topk_indices as topk
    w = dist.get_world_size(group)
    B, n = importance.shape
    if B % w:
        raise ValueError(f"topk_by_batch_shard: batch {B} is not a multiple of the {w} ranks")
    part = torch.empty((B // w, n), dtype=importance.dtype, device=importance.device)
    dist.reduce_scatter_tensor(part, importance.contiguous(), op=dist.ReduceOp.SUM, group=group)
    kept_part = topk(part, k).contiguous()
    kept = torch.empty((B, k), dtype=kept_part.dtype, device=kept_part.device)
    dist.all_gather_into_tensor(kept, kept_part, group=group)
    return kept, part
