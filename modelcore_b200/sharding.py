"""Batch sharding of independent decode rows over GPUs (one process per GPU).

Rows are independent sequences: no cache, attention or sampling state crosses rows, so the decode
path shards with no collective on its hot path.  Each rank owns a subset of the rows; the only
collective is a gather of the sampled token ids.

  contiguous_rows(n_rows, world, rank)  -> the rank's [begin, end) slice (equal-length rows)
  balanced_rows(lengths, world, equal_counts=False)
                                        -> per-rank row lists balancing the sum of context
                                           lengths (right-ragged prompts, e.g. lengths
                                           U[1024, 8192]): longest first onto the least-loaded
                                           rank; optionally the same row count on every rank
  gather_tokens(tokens, group=None)     -> every rank's (rows, steps) tokens concatenated in rank
                                           order (NCCL all_gather_into_tensor, or gloo all_gather)
"""
import heapq

import torch
import torch.distributed as dist


def contiguous_rows(n_rows, world, rank):
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    per, extra = divmod(n_rows, world)
    begin = rank * per + min(rank, extra)
    return begin, begin + per + (1 if rank < extra else 0)


def balanced_rows(lengths, world, equal_counts=False):
    """Greedy longest-processing-time assignment; each rank's rows come back sorted ascending.
    equal_counts=True also gives every rank the same number of rows (len(lengths) must be a
    multiple of world): a rank that holds its share leaves the pool.  Equal counts keep the
    per-rank token tensors one shape, as the gather needs."""
    n = len(lengths)
    if equal_counts and n % world:
        raise ValueError(f"{n} rows do not split into {world} equal shares")
    cap = n // world if equal_counts else n
    heap = [(0, r) for r in range(world)]
    out = [[] for _ in range(world)]
    for i in sorted(range(n), key=lambda i: (-int(lengths[i]), i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        if len(out[r]) < cap:
            heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(rows) for rows in out]


def gather_tokens(tokens, group=None):
    """Concatenates every rank's (rows, steps) int64 token tensor along rows, in rank order.
    All ranks must pass tensors of the same shape."""
    world = dist.get_world_size(group)
    if world == 1:
        return tokens
    if dist.get_backend(group) == "nccl":
        out = torch.empty((tokens.shape[0] * world,) + tuple(tokens.shape[1:]), dtype=tokens.dtype,
                          device=tokens.device)
        dist.all_gather_into_tensor(out, tokens.contiguous(), group=group)
        return out
    parts = [torch.empty_like(tokens) for _ in range(world)]
    dist.all_gather(parts, tokens.contiguous(), group=group)
    return torch.cat(parts, 0)
