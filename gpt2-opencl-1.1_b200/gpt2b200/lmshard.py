"""The LM head split over GPUs by vocabulary rows (optional, GPT-2 XL).

Every rank still decodes its own sequences with a full copy of the weights
(gpt2b200.replicas); only the last matvec of a step, the LM head
(main.c:1831: logits = LN_f(h) . wte^T over 50,257 rows), is shared out:

1. each rank runs its sequences' layers and final LayerNorm
   (Engine.decode_batch_rows);
2. the ranks all-gather those rows, so that every rank holds the rows of all
   ranks' sequences;
3. rank g computes the logits of every row over its range of vocabulary rows
   only (Engine.lm_head_rows: wte rows [v0, v1), a 1/n share of the head's
   bytes) and each row's first maximum there;
4. the ranks all-gather the per-row (value, index) pairs, and each rank keeps
   for its own rows the best over the ranges: the larger value, then the
   smaller index, which is the reference's first maximum over the whole
   vocabulary (main.c:1898-1904), so the tokens equal an unsplit head's.

Two collectives per step (NCCL on GPU ranks, gloo on CPU ranks for the tests)
replace reading all of wte on every rank.  The functions that need no GPU
(the ranges, the merge) are separate so that they can be tested on CPU ranks.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple


def vocab_range(vocab: int, world: int, rank: int, align: int = 128) -> Tuple[int, int]:
    """Vocabulary rows [v0, v1) of `rank`: contiguous shares, each boundary a
    multiple of `align` (whole feature tiles of the tensor-core GEMM); the
    last rank takes the remainder, and a rank past the end an empty range."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if vocab < 1 or align < 1:
        raise ValueError("vocabulary size and alignment must be positive")
    per = -(-vocab // world)
    per = -(-per // align) * align
    v0 = min(rank * per, vocab)
    return v0, min(v0 + per, vocab)


def merge_best(values, indices):
    """Per column, the best of the rows of (values, indices) [ranks, n]: the
    larger value, then the smaller index (first maximum).  torch tensors or
    anything torch.as_tensor takes; returns (values [n], indices [n])."""
    import torch
    v = torch.as_tensor(values)
    i = torch.as_tensor(indices).to(torch.int64)
    if v.ndim != 2 or v.shape != i.shape:
        raise ValueError("values and indices must both be [ranks, n]")
    best_v, best_i = v[0].clone(), i[0].clone()
    for g in range(1, v.shape[0]):
        take = (v[g] > best_v) | ((v[g] == best_v) & (i[g] < best_i))
        best_v = torch.where(take, v[g], best_v)
        best_i = torch.where(take, i[g], best_i)
    return best_v, best_i


def exchange_best(values, indices, own: slice):
    """All-gather each rank's per-row best over its vocabulary range and merge
    them for this rank's rows `own` (a slice of the gathered rows)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
    if world == 1:
        return merge_best(values[None, own], indices[None, own])
    gv = [torch.empty_like(values) for _ in range(world)]
    gi = [torch.empty_like(indices) for _ in range(world)]
    dist.all_gather(gv, values.contiguous())
    dist.all_gather(gi, indices.contiguous())
    return merge_best(torch.stack(gv)[:, own], torch.stack(gi)[:, own])


def gather_rows(rows):
    """All-gather every rank's rows [B, E] into [world * B, E], rank order."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
    if world == 1:
        return rows
    parts = [torch.empty_like(rows) for _ in range(world)]
    dist.all_gather(parts, rows.contiguous())
    return torch.cat(parts)


def generate_batch_sharded(eng, prompts: Sequence[Sequence[int]], n_new: int, device) -> List[List[int]]:
    """Greedy generation of this rank's sequences with the LM head split over
    the ranks of the default process group (every rank calls it with the same
    number of sequences and steps).  The first token of each sequence comes
    from its prefill (the full head, once); every later step runs steps 1-4
    above.  Returns n_new tokens per sequence, as generate_batch does."""
    import numpy as np
    import torch
    import torch.distributed as dist
    world = dist.get_world_size() if (dist.is_available() and dist.is_initialized()) else 1
    rank = dist.get_rank() if world > 1 else 0
    B = len(prompts)
    E, V = eng.cfg.n_embd, eng.cfg.vocab_size
    v0, v1 = vocab_range(V, world, rank)
    slots = np.arange(B, dtype=np.int32)
    toks = np.zeros(B, np.int32)
    pos = np.array([len(p) for p in prompts], np.int32)
    out = [[] for _ in range(B)]
    for s, p in enumerate(prompts):
        eng.prefill(np.asarray(p, np.int32), slot=s)
        toks[s] = eng.argmax(s)[0]
        out[s].append(int(toks[s]))
    rows = torch.empty((B, E), dtype=torch.float32, device=device)
    best_v = torch.empty(world * B, dtype=torch.float32, device=device)
    best_i = torch.empty(world * B, dtype=torch.int32, device=device)
    own = slice(rank * B, (rank + 1) * B)
    for _ in range(1, n_new):
        eng.decode_batch_rows(slots, toks, pos, rows)
        all_rows = gather_rows(rows)
        if world > 1 and all_rows.is_cuda:   # the engine's stream reads what torch's stream gathered
            torch.cuda.current_stream(all_rows.device).synchronize()
        if v1 > v0:
            eng.lm_head_rows(all_rows, world * B, v0, v1, best_v, best_i)
        else:   # a rank past the end of the vocabulary offers nothing
            best_v.fill_(float("-inf"))
            best_i.fill_(np.iinfo(np.int32).max)
        _, mine = exchange_best(best_v, best_i, own)
        toks = mine.to(torch.int32).cpu().numpy()
        pos += 1
        for s in range(B):
            out[s].append(int(toks[s]))
    return out
