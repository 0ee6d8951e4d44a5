"""Contiguous sharding of independent worlds across ranks (one GPU each).

Worlds never interact, so a step needs no communication: rank r of W owns
global worlds [N*r//W, N*(r+1)//W) and seeds them by global index, which
makes every world's trajectory independent of W.  The only collective is the
optional end-of-run reduction of diagnostics (NCCL over NVLink between GPUs,
gloo on CPU).
"""


def shard_range(n, rank, world_size):
    """[begin, end) of the worlds rank `rank` owns."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad rank %r of %r" % (rank, world_size))
    return n * rank // world_size, n * (rank + 1) // world_size


def world_stats(raw, caps):
    """Per-shard diagnostics (float64 [worlds, contacts, overflowed worlds,
    dropped contacts]) of a host copy of AoS worlds."""
    import numpy as np
    from . import layout
    v = layout.view(raw, caps)
    return np.array([len(v), v["contact_count"].sum(), (v["contact_overflow"] != 0).sum(),
                     v["contacts_dropped"].sum()], dtype=np.float64)


def reduce_stats(stats, device=None):
    """Sum a small stats vector over all ranks (no-op without a process group)."""
    import torch
    import torch.distributed as dist
    t = torch.as_tensor(stats, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().numpy()
