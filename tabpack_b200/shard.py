"""Member sharding over the GPUs of one box (one process per GPU, torch.distributed).

Members of a pack are independent (the training loss is a sum of per-member losses,
`src/tabpackage/_training.py:2679-2682`), so a pack shards by member with no gradient
exchange: rank r owns the contiguous global member range `ranges[r]`, dropout masks
and batch orders are keyed by global member id (shard-invariant), and the only
exchanges are the once-per-epoch all-gather of per-member validation predictions
(before greedy selection) and, at inference, a sum all-reduce of ensemble
probabilities.  When more models than pack slots are trained, freed slots take new
model ids in a fixed global order (`assign_replacements`).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


def member_ranges(n_members: int, world: int, cost: list[float] | None = None) -> list[tuple[int, int]]:
    """Contiguous member ranges, one per rank, in global member order.

    With `cost` (one number per member, e.g. its FLOPs per step) the cut points follow
    the cost prefix sums so that every rank gets about the same work; otherwise the
    counts differ by at most one.  Whenever `n_members >= world` every rank gets at
    least one member, however skewed the costs (a cut is clamped between one past the
    previous cut and the last position that still leaves a member for each later rank).
    """
    if world <= 0 or n_members < 0:
        raise ValueError('world must be positive and n_members non-negative')
    if cost is None:
        base, extra = divmod(n_members, world)
        out, start = [], 0
        for r in range(world):
            n = base + (1 if r < extra else 0)
            out.append((start, start + n))
            start += n
        return out
    if len(cost) != n_members:
        raise ValueError('one cost per member is required')
    total = float(sum(cost))
    prefix, acc = [], 0.0
    for c in cost:
        acc += float(c)
        prefix.append(acc)
    cuts = [0]
    for k in range(1, world):
        # first position whose prefix cost reaches the k-th share of the total
        i = next((j + 1 for j, s in enumerate(prefix) if s >= total * k / world), n_members)
        if n_members >= world:
            i = min(max(i, cuts[-1] + 1), n_members - (world - k))
        cuts.append(max(i, cuts[-1]))
    cuts.append(n_members)
    return [(cuts[k], cuts[k + 1]) for k in range(world)]


def gather_members(local: Tensor, counts: list[int], group=None) -> Tensor:
    """All-gather tensors with a leading member dimension from every rank and return
    them concatenated in global member order (ranks may own different counts)."""
    world = dist.get_world_size(group)
    if len(counts) != world:
        raise ValueError('one member count per rank is required')
    rank = dist.get_rank(group)
    if local.shape[0] != counts[rank]:
        raise ValueError('the local tensor does not match this rank\'s member count')
    maxc = max(counts)
    padded = local.new_zeros((maxc, *local.shape[1:]))
    padded[: local.shape[0]] = local
    if dist.get_backend(group) == 'nccl':
        out = local.new_empty((world * maxc, *local.shape[1:]))
        dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
        parts = [out[r * maxc: r * maxc + counts[r]] for r in range(world)]
    else:
        # host-side groups (gloo): device tensors are staged through host memory
        src = padded.cpu() if padded.is_cuda else padded.contiguous()
        bufs = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(bufs, src, group=group)
        parts = [bufs[r][: counts[r]].to(local.device) for r in range(world)]
    return torch.cat(parts, 0)


def allreduce_sum_(t: Tensor, group=None) -> Tensor:
    """In-place sum over ranks (ensemble probability partial sums)."""
    if t.is_cuda and dist.get_backend(group) != 'nccl':
        h = t.cpu()
        dist.all_reduce(h, op=dist.ReduceOp.SUM, group=group)
        t.copy_(h)
        return t
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def assign_replacements(stopped_slots: list[int], *, next_model_id: int, n_pending: int) -> list[tuple[int, int]]:
    """The replacement queue of a sharded pack (`src/tabpackage/_training.py:2891-2927`):
    (global slot, model id) pairs that refill the slots freed this epoch.

    As in the reference, the first `min(len(stopped_slots), n_pending)` freed slots in pack
    order take the next model ids in increasing order (`get_next_models`); the other freed
    slots stay empty.  Every rank derives `stopped_slots` from the same gathered validation
    metrics, so every rank computes the same pairs, and slot -- hence rank -- of a model does
    not depend on the number of GPUs."""
    if n_pending < 0 or next_model_id < 0:
        raise ValueError('n_pending and next_model_id must be non-negative')
    slots = sorted(stopped_slots)
    if len(set(slots)) != len(slots):
        raise ValueError('stopped slots must be distinct')
    n = min(len(slots), n_pending)
    return [(slots[i], next_model_id + i) for i in range(n)]
