"""Per-block deep-layer KV buffer (drop-in for utils/dynamic_block_kv.py).

Holds the current block's K/V per layer in BHSD [B, H_kv, block_size, D]
(same layout, dicts ``k`` / ``v`` keyed by layer, same methods as the
reference, utils/dynamic_block_kv.py:12-56).  ``write_full`` and ``write`` move
bytes with the append / row-scatter kernels; ``attend`` (new) runs the block
attention over cat(prefix, block) without materialising the concatenation.
"""
from __future__ import annotations

import torch

from .. import _lib
from .compaction import active_rows, compact_rows


class DynamicBlockKV:
    def __init__(self, deep_layer_start, num_layers, batch_size, num_kv_heads, block_size, head_dim, dtype, device):
        _lib.ensure_ops()
        self.deep_layer_start = deep_layer_start
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.block_size = block_size
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        self.k = {L: torch.zeros(batch_size, num_kv_heads, block_size, head_dim, dtype=dtype, device=device)
                  for L in range(deep_layer_start, num_layers)}
        self.v = {L: torch.zeros(batch_size, num_kv_heads, block_size, head_dim, dtype=dtype, device=device)
                  for L in range(deep_layer_start, num_layers)}
        self.batch_size = batch_size
        self._zero_start = torch.zeros(batch_size, dtype=torch.int32, device=device)

    def write_full(self, layer_idx, k, v):
        """Overwrite the whole block KV for a layer; k, v: [B, H_kv, block_size, D]."""
        # BHSD tensors viewed as [B, S, H, D] (strides carry the layout).
        torch.ops.fdl.kv_append([self.k[layer_idx].transpose(1, 2)], [self.v[layer_idx].transpose(1, 2)],
                                [k.transpose(1, 2)], [v.transpose(1, 2)], self._zero_start)

    def write(self, layer_idx, k, v, token_indices):
        """Scatter selected positions; k, v: [B, H_kv, n, D]; token_indices: [B, n]."""
        torch.ops.fdl.kv_scatter(self.k[layer_idx], self.v[layer_idx], k, v, token_indices.long(), 2)

    def get(self, layer_idx):
        return self.k[layer_idx], self.v[layer_idx]

    def reset(self):
        pass

    def compact_batch(self, active_indices):
        """Drop finished batch slots (utils/dynamic_block_kv.py:52-56) in
        place: every per-layer buffer keeps its storage and becomes a prefix
        view.  active_indices[i] must lie in [i, batch_size) -- any ascending
        list of distinct slots."""
        act = active_rows(active_indices, self.batch_size, self.device)
        n = act.numel()
        compact_rows(list(self.k.values()) + list(self.v.values()), act)
        for L in self.k:
            self.k[L] = self.k[L][:n]
            self.v[L] = self.v[L][:n]
        self.batch_size = n
        self._zero_start = self._zero_start[:n]
