"""In-place batch compaction shared by the cache classes.

The reference drops finished sequences with ``t[active_indices].contiguous()``
on every batch-indexed buffer (utils/static_kv_cache.py:350-398,
utils/dynamic_block_kv.py:52-56, utils/block_sparse_cache.py:141-147), which
allocates new tensors, so the caches cannot be compacted under CUDA graphs
(its docstring: "For CUDA graph mode, skip compaction").  Here the rows move
inside the existing storage with ``fdl_kv_compact`` (row i <- row
active_indices[i], in increasing i) and each buffer becomes a prefix view of
its old storage: data pointers do not change, so graphs captured for the
smaller batch read the right bytes, and ``restore_full_batch`` grows the views
back without allocating.
"""
from __future__ import annotations

from typing import Sequence

import torch


def active_rows(active_indices, batch: int, device) -> torch.Tensor:
    """Validate the reference's ``active_indices`` for in-place compaction and
    return them as a contiguous int64 tensor on ``device``.

    In place, row i can take row active_indices[i] only while that row is
    still unwritten, i.e. when i <= active_indices[i] < batch for every i.
    Every ascending list of distinct slots satisfies this -- in particular
    ``active_mask.nonzero()``, which is what the reference's samplers pass
    (utils/batch_bucketing.py:135).  Any other list raises ``ValueError``
    before anything moves.  The check reads one boolean back to the host; the
    reference's compaction is eager code at a block boundary as well.
    """
    act = torch.as_tensor(active_indices)
    if act.dtype == torch.bool:
        raise ValueError("compact_batch: active_indices must be integer slot indices, not a mask")
    act = act.reshape(-1).to(device=device, dtype=torch.int64).contiguous()
    n = act.numel()
    if n > batch:
        raise ValueError(f"compact_batch: {n} active slots for a batch of {batch}")
    if n:
        ok = (act >= torch.arange(n, device=act.device)) & (act < batch)
        if not bool(ok.all()):
            raise ValueError("compact_batch: in-place compaction needs i <= active_indices[i] < batch for every i "
                             "(an ascending list of distinct slots, as nonzero() returns); got "
                             f"{act.tolist()[:16]}")
    return act


def compact_rows(buffers: Sequence[torch.Tensor], act: torch.Tensor) -> None:
    """Move row act[i] to row i in every buffer (one launch per 128 buffers
    of the same row size and batch stride)."""
    bufs = [b for b in buffers if b is not None]
    if bufs and act.numel():
        torch.ops.fdl.kv_compact(bufs, act)


def regrow(t: torch.Tensor, rows: int, dim: int = 0) -> torch.Tensor:
    """Zeroed view of ``t`` with ``rows`` entries along ``dim`` over the same
    storage -- the full-batch buffer that compaction turned into a prefix view
    -- or new zeros when that storage is smaller than the full shape."""
    shape = list(t.shape)
    shape[dim] = rows
    try:
        full = t.as_strided(shape, t.stride(), t.storage_offset())
    except RuntimeError:
        return torch.zeros(shape, dtype=t.dtype, device=t.device)
    return full.zero_()
