"""Request sharding across the GPUs of one box.

The MiniPrefix forward has no exchange step between requests: every GPU holds a
replica of the weights, its own K/V page pool, block tables, prefix cache,
scheduler and engine (one process per GPU), and a request lives on one GPU for
its whole life. Scaling is therefore a deterministic routing decision on the
host, made identically by every rank from the same global request list, with no
collective on the data path:

* ``round_robin`` -- request i goes to rank i % world (uniform workloads such as
  BASELINE configs 3 and 4, where every request carries the same work);
* ``by_root`` -- requests drawn from a prefix tree go to the rank that owns their
  root (roots dealt round-robin over ranks), so all requests that can share
  cached pages meet the same prefix cache (16 roots, 2 per GPU
  at 8 GPUs).

Within a rank the global submission order is kept, so each shard's bookkeeping is
exactly what the reference engine does when it is given that shard's requests in
that order. ``gather_counters`` sums per-rank counters once, after the timed
region (host-side reporting, not part of a step).
"""
from __future__ import annotations

from typing import Sequence


def round_robin(count: int, world: int, rank: int) -> list[int]:
    """Global indices of the requests rank `rank` serves, in submission order."""
    _check(world, rank)
    if count < 0:
        raise ValueError("negative request count")
    return list(range(rank, count, world))


def by_root(roots: Sequence[int], world: int, rank: int) -> list[int]:
    """Global indices of the requests whose prefix-tree root this rank owns. The
    distinct root ids, sorted ascending, are dealt round-robin over the ranks, so
    the split does not depend on the order of the requests."""
    _check(world, rank)
    owner = {r: i % world for i, r in enumerate(sorted(set(int(x) for x in roots)))}
    return [i for i, r in enumerate(roots) if owner[int(r)] == rank]


def partition(count_or_roots, world: int, policy: str = "round_robin") -> list[list[int]]:
    """Every rank's request list (the whole routing table, as each rank computes it)."""
    if policy == "round_robin":
        return [round_robin(int(count_or_roots), world, r) for r in range(world)]
    if policy == "by_root":
        return [by_root(count_or_roots, world, r) for r in range(world)]
    raise ValueError(f"unknown routing policy {policy!r}")


def gather_counters(values: dict, dist=None) -> dict:
    """Sum of every rank's integer/float counters (all ranks get the result). With
    no process group (one GPU) the input is returned unchanged."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return dict(values)
    import torch

    keys = sorted(values)
    backend = dist.get_backend()
    device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(values[k]) for k in keys], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return {k: (int(v) if isinstance(values[k], int) else float(v)) for k, v in zip(keys, t.cpu().tolist())}


def _check(world: int, rank: int) -> None:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
