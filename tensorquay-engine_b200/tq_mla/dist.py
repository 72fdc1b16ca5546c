"""Multi-device paged MLA: request sharding and the cross-device KV split of long contexts.

Two strategies, one process per GPU:
  - request sharding (``inputs.shard``): whole sequences are assigned to devices by token count;
    each device owns the pages of its sequences and runs the kernel on them; no collective is
    on the data path.
  - context split (``context_split`` + ``gather_merge``): for very long single-token decodes,
    every device holds a contiguous, page-aligned range of each sequence's positions and
    computes a partial result (f32 output normalised over its range, natural-log lse); the
    partials are all-gathered (``torch.distributed`` over NCCL) and merged by log-sum-exp with
    ``tq_mla_combine``. The reference plans this as decode context parallelism
    (docs/ARCHITECTURE.md:240-241,313).
"""

import numpy as np

from . import inputs

PAGE_ROWS = 64


def context_ranges(kv_len, world):
    """Page-aligned position ranges ``[(start, end)] * world`` for one sequence of ``kv_len``."""
    pages = (int(kv_len) + PAGE_ROWS - 1) // PAGE_ROWS
    cuts = [(pages * r) // world for r in range(world + 1)]
    return [(min(kv_len, cuts[r] * PAGE_ROWS), min(kv_len, cuts[r + 1] * PAGE_ROWS))
            for r in range(world)]


def context_split(w: inputs.Workload, world: int, rank: int) -> inputs.Workload:
    """This device's share of a single-token decode batch: positions ``[a_r, b_r)`` of each
    sequence, as sequences of their own (cache contents keep their global data offsets)."""
    if (w.q_per_seq != 1).any():
        raise ValueError("the context split applies to single-token decode")
    if ((w.prefix + 1) < w.kv_len).any():
        raise ValueError("the context split needs every cached position to be visible")
    starts, lens = [], []
    for n in w.kv_len:
        a, b = context_ranges(int(n), world)[rank]
        starts.append(a)
        lens.append(b - a)
    starts = np.asarray(starts, dtype=np.int64)
    lens = np.asarray(lens, dtype=np.int64)
    tok_off = np.concatenate([[0], np.cumsum(w.kv_len)[:-1]]).astype(np.int64) + starts
    sub = inputs.Workload(f"{w.name} context part {rank}/{world}", w.seed, w.heads, w.width, lens,
                          w.q_per_seq.copy(), lens - 1, w.scale,
                          seq_global=np.arange(w.sequences),
                          token_global=np.arange(w.sequences, dtype=np.int64),
                          tok_off_global=tok_off)
    return inputs._finish(sub)


def gather_merge(part_out, part_lse, group=None, out=None, lse=None):
    """All-gather per-device partials (``f32 [T,H,512]``, ``f32 [T,H]``) and merge them.

    On GPUs the merge runs in ``tq_mla_combine``; on CPU tensors (gloo) it is left to the caller
    (returns the gathered stacks), since there is no CPU compute path.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    g_out = torch.empty((world, *part_out.shape), dtype=part_out.dtype, device=part_out.device)
    g_lse = torch.empty((world, *part_lse.shape), dtype=part_lse.dtype, device=part_lse.device)
    if part_out.is_cuda:
        dist.all_gather_into_tensor(g_out, part_out.contiguous(), group=group)
        dist.all_gather_into_tensor(g_lse, part_lse.contiguous(), group=group)
        from .ops import combine_parts

        return combine_parts(g_out, g_lse, out=out, lse=lse)
    dist.all_gather(list(g_out.unbind(0)), part_out.contiguous(), group=group)
    dist.all_gather(list(g_lse.unbind(0)), part_lse.contiguous(), group=group)
    return g_out, g_lse
