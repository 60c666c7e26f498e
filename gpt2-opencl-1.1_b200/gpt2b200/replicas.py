"""Independent-sequence replicas across ranks (one process per GPU).

GPT-2 fits on one GPU and sequences never interact, so the multi-GPU path
shards *sequences*, not tensors: rank r of n holds a full copy of the weights
and decodes its own block of sequences; nothing crosses ranks on the data path.
The host side needs only three things, kept here so that they can be tested on
CPU ranks (gloo) as well as run on GPU ranks (NCCL):

* ``shard``: which global sequences a rank owns -- rank g gets the contiguous
  block [g*B/n, (g+1)*B/n) of B sequences (strong scaling: B fixed), or B per
  rank (weak scaling: B*n in total);
* ``max_over_ranks``: the job's time is the slowest rank's;
* ``gather_streams``: rank 0 collects every sequence's token stream in global
  order (the host-side gather of the reference's single-sequence loop,
  main.c:2108-2140, generalised to many sequences).
"""
from __future__ import annotations

from typing import Callable, List, Sequence


def shard(n_seq: int, world: int, rank: int, scaling: str = "strong") -> List[int]:
    """Global sequence indices owned by `rank`.

    strong: `n_seq` sequences in total split into contiguous blocks (the first
    n_seq % world ranks get one more); weak: `n_seq` sequences on every rank.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if n_seq < 0:
        raise ValueError("negative sequence count")
    if scaling == "weak":
        return list(range(rank * n_seq, (rank + 1) * n_seq))
    if scaling != "strong":
        raise ValueError(f"unknown scaling {scaling!r}")
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def max_over_ranks(values: Sequence[float], device=None) -> List[float]:
    """Element-wise max over all ranks (identity without an initialised process group)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def gather_streams(local: dict, dst: int = 0):
    """Collect {global sequence index: token list} from every rank on `dst`.

    Returns the streams ordered by global index on `dst`, None elsewhere.
    """
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [list(map(int, local[k])) for k in sorted(local)]
    world, rank = dist.get_world_size(), dist.get_rank()
    parts = [None] * world if rank == dst else None
    dist.gather_object({int(k): list(map(int, v)) for k, v in local.items()}, parts, dst=dst)
    if rank != dst:
        return None
    merged = {}
    for p in parts:
        for k, v in p.items():
            if k in merged:
                raise RuntimeError(f"sequence {k} decoded by two ranks")
            merged[k] = v
    return [merged[k] for k in sorted(merged)]


def run_replica(generate: Callable[[list], list], prompts: Callable[[int], Sequence[int]], n_seq: int,
                scaling: str = "strong") -> dict:
    """Decode this rank's sequences with `generate(list_of_prompts) -> list_of_streams`.

    `prompts(i)` gives the prompt of global sequence i, so a sequence's tokens
    do not depend on how many ranks share the job.
    """
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(), dist.get_rank()
    else:
        world, rank = 1, 0
    mine = shard(n_seq, world, rank, scaling)
    if not mine:
        return {}
    streams = generate([list(prompts(i)) for i in mine])
    if len(streams) != len(mine):
        raise RuntimeError(f"generate returned {len(streams)} streams for {len(mine)} prompts")
    return dict(zip(mine, streams))
