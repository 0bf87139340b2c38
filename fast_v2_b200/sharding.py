"""Sequence sharding across GPUs (one process per GPU).

The KV-cache path is batch-row local -- every cache op reads and writes only
its own sequence's rows (utils/static_kv_cache.py:228, 246;
utils/dynamic_block_kv.py:41-43) -- so a multi-GPU job shards the requests by
sequence, each rank holding a full weight replica and its own KV cache, with no
collective on the data path.  The reference does the same at the request level
(lm-eval rank sharding under accelerate, eval.py:141-150).  The only
collectives are after decoding: one all-gather of the generated token ids and
a max-reduction of the per-rank device time.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def sequence_shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first, count) of the contiguous run of sequences owned by `rank` when
    `total` sequences are split as evenly as possible over `world` ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def _device_for(group=None) -> torch.device:
    backend = dist.get_backend(group)
    return torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")


def gather_generated(tokens: torch.Tensor, pad_id: int, group=None) -> torch.Tensor:
    """All-gather every rank's generated ids [n_local, L] (int64) into
    [sum(n_local), L_max]; shorter shards and rows are padded with pad_id.
    Every rank receives the whole result."""
    world = dist.get_world_size(group)
    dev = _device_for(group)
    n, L = tokens.shape
    sizes = torch.tensor([n, L], dtype=torch.int64, device=dev)
    all_sizes = torch.empty(world * 2, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(all_sizes, sizes, group=group)
    all_sizes = all_sizes.view(world, 2)
    n_max, l_max = (int(x) for x in all_sizes.max(dim=0).values)
    buf = torch.full((n_max, l_max), pad_id, dtype=torch.int64, device=dev)
    buf[:n, :L] = tokens.to(dev)
    out = torch.empty(world * n_max, l_max, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(out, buf, group=group)
    keep = torch.cat([torch.arange(r * n_max, r * n_max + int(all_sizes[r, 0]), device=dev) for r in range(world)])
    return out.index_select(0, keep)


def max_over_ranks(value: float, group=None) -> float:
    """Maximum of a per-rank scalar (e.g. device milliseconds) over the group."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=_device_for(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
