"""Data-parallel plumbing for the 800h decode across the GPUs of one node: every sequence's decode reads only its own
pages, so sequences are sharded over ranks and nothing crosses NVLink on the decode path.  Collectives appear only
around it: the max-over-ranks step time and, for checking, gathering the per-rank outputs to rank 0.

Works with any torch.distributed backend (nccl on GPUs, gloo on CPU for tests)."""
import heapq

import torch
import torch.distributed as dist


def row_cost(n, win=0):
    """Bytes one decode of a row of n tokens reads (the reference's formula, nvidia/check_nvidia.py:563)."""
    if win:
        return (min(n, win) + 4) * 2048
    nq = max(0, n - 128) // 256
    return nq * 256 * 200 + (n - nq * 256) * 2048


def shard_rows(lengths, world, rank, win=0):
    """Rows of `lengths` assigned to `rank`: longest-processing-time greedy over the rows' read bytes, so every rank
    gets about the same bytes (ties broken by row index, identical on every rank).  Returns sorted row indices."""
    order = sorted(range(len(lengths)), key=lambda i: (-row_cost(lengths[i], win), i))
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(lengths)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + row_cost(lengths[i], win), r))
    return [i for i in range(len(lengths)) if owner[i] == rank]


def max_over_ranks(seconds, device=None):
    """The largest value of `seconds` over all ranks (the step time of a data-parallel job)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(seconds)
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(out, rows, total, device=None):
    """Gather per-rank outputs (len(rows), ...) to rank 0 into a (total, ...) tensor ordered by global row index;
    other ranks get None.  Shapes are padded to the largest shard so the collective is a plain all_gather."""
    world = dist.get_world_size()
    n = torch.tensor([len(rows)], dtype=torch.int64, device=device)
    ns = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(ns, n)
    m = int(max(x.item() for x in ns))
    pad = torch.zeros((m,) + tuple(out.shape[1:]), dtype=out.dtype, device=device)
    pad[:len(rows)] = out
    idx = torch.full((m,), -1, dtype=torch.int64, device=device)
    idx[:len(rows)] = torch.as_tensor(rows, dtype=torch.int64, device=device)
    # the rows travel as their bytes: NCCL moves no int16 / uint16 tensors, and a byte copy is exact for any dtype
    raw = pad.contiguous().view(torch.uint8)
    outs = [torch.zeros_like(raw) for _ in range(world)]
    idxs = [torch.zeros_like(idx) for _ in range(world)]
    dist.all_gather(outs, raw)
    dist.all_gather(idxs, idx)
    outs = [o.view(out.dtype) for o in outs]
    if dist.get_rank() != 0:
        return None
    full = torch.zeros((total,) + tuple(out.shape[1:]), dtype=out.dtype, device=device)
    for o, ix in zip(outs, idxs):
        keep = ix >= 0
        full[ix[keep]] = o[keep]
    return full
