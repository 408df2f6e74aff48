"""Work partitioning across the GPUs of one node.

* Batches shard by sequence (no collective): LPT on token counts.
* One long sequence shards by KV range: contiguous page-aligned ranges, one
  per rank; each rank produces the partial (m, l, o) of its range and the
  root merges them (qwanto_b200.merge_partials / the NCCL gather in
  :func:`gather_and_merge`).
"""
from __future__ import annotations

from typing import List, Sequence


def lpt_shard(tokens: Sequence[int], ranks: int) -> List[List[int]]:
    """Longest-processing-time partition of sequence indices by token count.

    Deterministic: ties broken by sequence index, then by the lowest rank.
    Each rank's list is returned in ascending sequence order."""
    if ranks <= 0:
        raise ValueError("ranks must be positive")
    order = sorted(range(len(tokens)), key=lambda i: (-int(tokens[i]), i))
    load = [0] * ranks
    parts: List[List[int]] = [[] for _ in range(ranks)]
    for i in order:
        r = min(range(ranks), key=lambda k: (load[k], len(parts[k]), k))
        parts[r].append(i)
        load[r] += int(tokens[i])
    return [sorted(p) for p in parts]


def balanced_count_shard(tokens: Sequence[int], ranks: int) -> List[List[int]]:
    """LPT restricted to an equal number of sequences per rank (weak scaling
    keeps the per-GPU batch fixed): sequences sorted by length are dealt in
    boustrophedon order, which balances both count and tokens."""
    n = len(tokens)
    if n % ranks:
        raise ValueError("sequence count must divide by the rank count")
    order = sorted(range(n), key=lambda i: (-int(tokens[i]), i))
    parts: List[List[int]] = [[] for _ in range(ranks)]
    for k, i in enumerate(order):
        rnd, pos = divmod(k, ranks)
        r = pos if rnd % 2 == 0 else ranks - 1 - pos
        parts[r].append(i)
    return [sorted(p) for p in parts]


def kv_ranges(total_tokens: int, ranks: int, page_tokens: int) -> List[tuple]:
    """Split [0, total_tokens) into `ranks` contiguous page-aligned ranges of
    nearly equal size; the last rank also owns the tail (where appends go)."""
    pages = (total_tokens + page_tokens - 1) // page_tokens
    out = []
    for r in range(ranks):
        p0 = pages * r // ranks
        p1 = pages * (r + 1) // ranks
        out.append((min(p0 * page_tokens, total_tokens), min(p1 * page_tokens, total_tokens)))
    return out


def merge_partials_host(m, l, o):
    """Reference merge of base-2 partial states on the host (numpy):
    m*, l* = max m, sum l 2^(m-m*); out = sum o 2^(m-m*) / l*."""
    import numpy as np
    m = np.asarray(m, np.float64)
    l = np.asarray(l, np.float64)
    o = np.asarray(o, np.float64)
    ms = m.max(axis=0)
    w = np.where(np.isneginf(m), 0.0, np.exp2(m - ms))
    ls = (l * w).sum(axis=0)
    return (o * w[..., None]).sum(axis=0) / np.where(ls > 0, ls, 1.0)[..., None]


def gather_and_merge(m, l, o, out, rows: int, group=None):
    """All-gather the per-rank partial (m, l, o) with torch.distributed and
    merge on every rank with the library's merge kernel (CUDA tensors) or
    numpy (CPU tensors, used by the gloo tests)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    ms = [torch.empty_like(m) for _ in range(world)]
    ls = [torch.empty_like(l) for _ in range(world)]
    os_ = [torch.empty_like(o) for _ in range(world)]
    dist.all_gather(ms, m, group=group)
    dist.all_gather(ls, l, group=group)
    dist.all_gather(os_, o, group=group)
    M, L, O = torch.stack(ms), torch.stack(ls), torch.stack(os_)
    if M.is_cuda:
        from . import merge_partials
        merge_partials(world, rows, M, L, O, out)
    else:
        out.copy_(torch.from_numpy(merge_partials_host(M.numpy(), L.numpy(), O.numpy())).float())
    return out
