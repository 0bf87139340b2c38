"""Block-level sparse cache for token-sparse diffusion (drop-in for
utils/block_sparse_cache.py).

Four stacked [L, B, block_size, hidden] caches with the reference's methods
(utils/block_sparse_cache.py:19-147).  ``scatter_attn_output`` /
``scatter_mlp_output`` use the row-scatter kernel on [B, n] block positions
instead of ``scatter_`` with an expanded int64 index.
"""
from __future__ import annotations

import torch

from .. import _lib
from .compaction import active_rows, compact_rows


class BlockSparseCache:
    def __init__(self, num_layers: int, batch_size: int, block_size: int, hidden_size: int, dtype: torch.dtype,
                 device: torch.device):
        _lib.ensure_ops()
        self.num_layers = num_layers
        self.batch_size = batch_size
        self.block_size = block_size
        self.hidden_size = hidden_size
        self.dtype = dtype
        self.device = device
        shape = (num_layers, batch_size, block_size, hidden_size)
        self.layer_input = torch.zeros(shape, dtype=dtype, device=device)
        self.attn_output = torch.zeros(shape, dtype=dtype, device=device)
        self.mlp_input = torch.zeros(shape, dtype=dtype, device=device)
        self.mlp_output = torch.zeros(shape, dtype=dtype, device=device)

    def cache_layer_input(self, layer_idx: int, hidden_states: torch.Tensor):
        self.layer_input.select(0, layer_idx).copy_(hidden_states)

    def cache_attn_output(self, layer_idx: int, attn_out: torch.Tensor):
        self.attn_output.select(0, layer_idx).copy_(attn_out)

    def cache_mlp_input(self, layer_idx: int, mid: torch.Tensor):
        self.mlp_input.select(0, layer_idx).copy_(mid)

    def cache_mlp_output(self, layer_idx: int, mlp_out: torch.Tensor):
        self.mlp_output.select(0, layer_idx).copy_(mlp_out)

    def get_layer_input(self, layer_idx: int) -> torch.Tensor:
        return self.layer_input.select(0, layer_idx)

    def get_attn_output(self, layer_idx: int) -> torch.Tensor:
        return self.attn_output.select(0, layer_idx)

    def get_mlp_input(self, layer_idx: int) -> torch.Tensor:
        return self.mlp_input.select(0, layer_idx)

    def get_mlp_output(self, layer_idx: int) -> torch.Tensor:
        return self.mlp_output.select(0, layer_idx)

    def scatter_attn_output(self, layer_idx: int, token_indices: torch.Tensor, values: torch.Tensor):
        torch.ops.fdl.kv_scatter(self.attn_output.select(0, layer_idx), None, values, None, token_indices.long(), 1)

    def scatter_mlp_output(self, layer_idx: int, token_indices: torch.Tensor, values: torch.Tensor):
        torch.ops.fdl.kv_scatter(self.mlp_output.select(0, layer_idx), None, values, None, token_indices.long(), 1)

    def reset(self):
        pass

    def compact_batch(self, active_indices: torch.Tensor):
        """Drop finished batch slots (utils/block_sparse_cache.py:141-147) in
        place: the four [L, B, block, hidden] buffers keep their storage and
        become [L, n, block, hidden] views (each layer's slice stays
        contiguous).  active_indices[i] must lie in [i, batch_size) -- any
        ascending list of distinct slots."""
        act = active_rows(active_indices, self.batch_size, self.device)
        n = act.numel()
        bufs = (self.layer_input, self.attn_output, self.mlp_input, self.mlp_output)
        compact_rows([t.select(0, l) for t in bufs for l in range(self.num_layers)], act)
        self.layer_input, self.attn_output, self.mlp_input, self.mlp_output = (t[:, :n] for t in bufs)
        self.batch_size = n
