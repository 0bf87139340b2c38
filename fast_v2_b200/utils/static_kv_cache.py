"""Static KV caches for Fast-dLLM v2 block diffusion, backed by sm_100a kernels.

Drop-in for utils/static_kv_cache.py of the reference: same classes, same
constructor arguments, attributes and methods, same BSHD per-layer buffers
(``key_cache[l]`` / ``value_cache[l]`` of shape [B, max_seq_len, H_kv, D]),
same device control tensors (``cache_seqlens``, ``scratch_seqlens``,
``kv_write_start``).  What changes is how the writes move bytes:

* commit ``update`` / ``write_scratch_compiled`` / ``write_scratch`` call the
  append kernel (16-byte vector copies with a per-sequence start held in a
  device int32 [B] buffer) instead of slice ``copy_`` or ``scatter_`` with a
  full-shape int64 index (the reference's index alone is 4x the data bytes,
  utils/static_kv_cache.py:205-216);
* ``write_sparse`` calls the row-scatter kernel on the [B, n] positions;
* ``append`` (new) takes per-sequence start positions, so sequences of a
  batch may hold different committed lengths;
* ``gather_prefix`` (new) packs the valid prefix of every sequence, optionally
  GQA-expanded, into a varlen buffer.

All kernels launch on torch's current stream and allocate nothing, so the
methods stay CUDA-graph capturable and traceable by torch.compile (the ops
have Meta kernels).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _lib
from .compaction import active_rows, compact_rows, regrow


def _mark(t: torch.Tensor) -> None:
    try:
        torch._dynamo.mark_static_address(t)
    except Exception:  # pragma: no cover - dynamo unavailable
        pass


class StaticKVCache:
    """Cross-block KV cache (reference: utils/static_kv_cache.py:19-398)."""

    def __init__(
        self,
        batch_size: int,
        max_seq_len: int,
        num_layers: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device,
    ):
        _lib.ensure_ops()
        self.batch_size = batch_size
        self.max_batch_size = batch_size
        self.max_seq_len = max_seq_len
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        self.key_cache = [
            torch.zeros(batch_size, max_seq_len, num_kv_heads, head_dim, dtype=dtype, device=device)
            for _ in range(num_layers)
        ]
        self.value_cache = [
            torch.zeros(batch_size, max_seq_len, num_kv_heads, head_dim, dtype=dtype, device=device)
            for _ in range(num_layers)
        ]
        self._seq_len = 0
        self.cache_seqlens = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self.scratch_seqlens = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self.kv_write_start = torch.zeros((), dtype=torch.int64, device=device)
        self._write_idx = torch.zeros(max_seq_len, dtype=torch.int64, device=device)
        self._arange = torch.arange(max_seq_len, dtype=torch.int64, device=device)
        self._attn_mask_buffer = torch.zeros(batch_size, 1, 1, max_seq_len, dtype=dtype, device=device)
        self._kv_indices = torch.arange(max_seq_len, dtype=torch.int32, device=device)
        # Append start positions (int32 [B]) for the commit path and for the
        # scratch path; filled from eager code, read by the append kernel.
        self._commit_start = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self._scratch_start = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self._commit_start_value = 0
        self._write_idx_fixed = None
        self._mark_static_addresses()

    def _mark_static_addresses(self):
        for layer_idx in range(self.num_layers):
            _mark(self.key_cache[layer_idx])
            _mark(self.value_cache[layer_idx])
        for t in (self.cache_seqlens, self.scratch_seqlens, self.kv_write_start, self._write_idx, self._arange,
                  self._attn_mask_buffer, self._kv_indices, self._commit_start, self._scratch_start):
            _mark(t)

    # ------------------------------------------------------------------
    # DynamicCache-compatible interface (eager prefill / commit)
    # ------------------------------------------------------------------
    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """Append [B, S, H, D] at the committed length (all sequences), advance
        after the last layer (utils/static_kv_cache.py:132-160)."""
        seq_len = key_states.shape[1]
        start = self._seq_len
        if start + seq_len > self.max_seq_len:
            raise ValueError(f"StaticKVCache.update: {start}+{seq_len} exceeds max_seq_len={self.max_seq_len}")
        if self._commit_start_value != start:
            self._commit_start.fill_(start)
            self._commit_start_value = start
        torch.ops.fdl.kv_append([self.key_cache[layer_idx]], [self.value_cache[layer_idx]], [key_states],
                                [value_states], self._commit_start)
        if layer_idx == self.num_layers - 1:
            self._seq_len += seq_len
            self.cache_seqlens.fill_(self._seq_len)
        end = start + seq_len
        return self.key_cache[layer_idx][:, :end], self.value_cache[layer_idx][:, :end]

    def __getitem__(self, layer_idx):
        end = self._seq_len
        return self.key_cache[layer_idx][:, :end], self.value_cache[layer_idx][:, :end]

    def __len__(self):
        return self.num_layers if self._seq_len > 0 else 0

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._seq_len

    # ------------------------------------------------------------------
    # Per-sequence lengths (new)
    # ------------------------------------------------------------------
    def append(self, key_states, value_states, layer_idx, start_pos: torch.Tensor):
        """Append [B, S, H, D] at per-sequence positions start_pos (device
        int32 [B]); does not move any length pointer."""
        torch.ops.fdl.kv_append([self.key_cache[layer_idx]], [self.value_cache[layer_idx]], [key_states],
                                [value_states], start_pos)

    def append_layers(self, key_states: list, value_states: list, start_pos: torch.Tensor):
        """Append one block for every layer in a single launch."""
        torch.ops.fdl.kv_append(self.key_cache, self.value_cache, list(key_states), list(value_states), start_pos)

    def gather_prefix(self, layer_idx, lens: torch.Tensor, cu_seqlens: torch.Tensor, k_out, v_out, n_rep: int = 1):
        """Pack cache[b, :lens[b]] for every b into k_out/v_out
        [sum(lens), H*n_rep, D] (GQA-expanded when n_rep > 1)."""
        torch.ops.fdl.kv_gather_prefix(self.key_cache[layer_idx], self.value_cache[layer_idx], lens, None, None, n_rep,
                                       k_out, v_out, cu_seqlens, 1, 1)

    # ------------------------------------------------------------------
    # Compiled-graph-friendly methods (tensor control inputs only)
    # ------------------------------------------------------------------
    def prepare_write_idx(self, seq_len: int):
        """Stage the scratch write position (kv_write_start) for
        write_scratch_compiled (utils/static_kv_cache.py:180-216).  Device ops
        only; the append kernel needs no expanded index tensor."""
        if self._write_idx_fixed is None or self._write_idx_fixed.shape[0] != seq_len:
            self._write_idx_fixed = torch.zeros(seq_len, dtype=torch.int64, device=self.device)
            _mark(self._write_idx_fixed)
        self._write_idx_fixed.copy_(self._arange[:seq_len] + self.kv_write_start)
        self._scratch_start.copy_(self.kv_write_start.expand(self.batch_size))

    def write_scratch_compiled(self, key_states, value_states, layer_idx):
        """Write the current block at kv_write_start without advancing the
        committed length (utils/static_kv_cache.py:218-229)."""
        torch.ops.fdl.kv_append([self.key_cache[layer_idx]], [self.value_cache[layer_idx]], [key_states],
                                [value_states], self._scratch_start)

    def write_sparse(self, key_states, value_states, layer_idx, write_positions):
        """K/V rows at per-batch absolute positions [B, n]
        (utils/static_kv_cache.py:231-247)."""
        torch.ops.fdl.kv_scatter(self.key_cache[layer_idx], self.value_cache[layer_idx], key_states, value_states,
                                 write_positions.long(), 1)

    def get_full_kv(self, layer_idx):
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def set_scratch_seqlens(self, total_valid_len: int):
        self.scratch_seqlens.fill_(total_valid_len)

    def set_kv_write_start(self, offset: int):
        self.kv_write_start.fill_(offset)

    # ------------------------------------------------------------------
    # Legacy methods (eager only)
    # ------------------------------------------------------------------
    def write_scratch(self, key_states, value_states, layer_idx, position):
        start = torch.full((self.batch_size,), int(position), dtype=torch.int32, device=self.device)
        torch.ops.fdl.kv_append([self.key_cache[layer_idx]], [self.value_cache[layer_idx]], [key_states],
                                [value_states], start)

    def get_kv_up_to(self, layer_idx, length):
        return self.key_cache[layer_idx][:, :length], self.value_cache[layer_idx][:, :length]

    def get_seqused_mask(self, total_valid_len: int):
        self._attn_mask_buffer.fill_(0.0)
        invalid = self._kv_indices[None, :] >= total_valid_len
        self._attn_mask_buffer.masked_fill_(invalid[:, None, None, :], float("-inf"))
        return self._attn_mask_buffer

    def get_seqused_mask_batched(self, seqused: torch.Tensor):
        self._attn_mask_buffer.fill_(0.0)
        invalid = self._kv_indices[None, :] >= seqused[:, None]
        self._attn_mask_buffer.masked_fill_(invalid[:, None, None, :], float("-inf"))
        return self._attn_mask_buffer

    def reset(self):
        self._seq_len = 0
        self.cache_seqlens.fill_(0)

    def zero_and_reset(self):
        for layer_idx in range(self.num_layers):
            self.key_cache[layer_idx].zero_()
            self.value_cache[layer_idx].zero_()
        self._seq_len = 0
        self.cache_seqlens.fill_(0)
        self.scratch_seqlens.fill_(0)
        self.kv_write_start.fill_(0)

    def restore_full_batch(self):
        """Back to max_batch_size after compact_batch (utils/static_kv_cache.py:
        319-348): the prefix views grow back over their own storage, zeroed as
        the reference's fresh buffers are, so data pointers do not change."""
        if self.batch_size == self.max_batch_size:
            return
        bs = self.max_batch_size
        self.key_cache = [regrow(t, bs) for t in self.key_cache]
        self.value_cache = [regrow(t, bs) for t in self.value_cache]
        self.cache_seqlens = regrow(self.cache_seqlens, bs)
        self.scratch_seqlens = regrow(self.scratch_seqlens, bs)
        self._attn_mask_buffer = regrow(self._attn_mask_buffer, bs)
        self._commit_start = regrow(self._commit_start, bs)
        self._scratch_start = regrow(self._scratch_start, bs)
        self._commit_start_value = 0
        self._seq_len = 0
        self.kv_write_start.fill_(0)
        self.batch_size = bs

    def compact_batch(self, active_indices: torch.Tensor):
        """Drop finished batch slots (utils/static_kv_cache.py:350-398) in
        place: row i of every batch-indexed buffer takes row
        active_indices[i], then each buffer becomes a prefix view of its own
        storage, so data pointers stay valid for CUDA graphs.
        active_indices[i] must lie in [i, batch_size) for every i -- any
        ascending list of distinct slots, as ``nonzero()`` returns; other
        lists raise ValueError."""
        act = active_rows(active_indices, self.batch_size, self.device)
        n = act.numel()
        compact_rows(self.key_cache + self.value_cache, act)
        compact_rows([self.cache_seqlens, self.scratch_seqlens, self._commit_start, self._scratch_start], act)
        self.key_cache = [t[:n] for t in self.key_cache]
        self.value_cache = [t[:n] for t in self.value_cache]
        self.cache_seqlens = self.cache_seqlens[:n]
        self.scratch_seqlens = self.scratch_seqlens[:n]
        self._commit_start = self._commit_start[:n]
        self._scratch_start = self._scratch_start[:n]
        self._write_idx_fixed = None
        self._attn_mask_buffer = self._attn_mask_buffer[:n].zero_()
        self.batch_size = n


class StaticBlockCache:
    """Within-block sub-block cache [B, block_size, H, D] per layer
    (reference: utils/static_kv_cache.py:401-491)."""

    def __init__(self, batch_size: int, block_size: int, num_layers: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device):
        _lib.ensure_ops()
        self.batch_size = batch_size
        self.block_size = block_size
        self.num_layers = num_layers
        self.dtype = dtype
        self.device = device
        self.key_cache = [torch.zeros(batch_size, block_size, num_kv_heads, head_dim, dtype=dtype, device=device)
                          for _ in range(num_layers)]
        self.value_cache = [torch.zeros(batch_size, block_size, num_kv_heads, head_dim, dtype=dtype, device=device)
                            for _ in range(num_layers)]
        self._zero_start = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self._num_initialized = 0
        for layer_idx in range(num_layers):
            _mark(self.key_cache[layer_idx])
            _mark(self.value_cache[layer_idx])

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        torch.ops.fdl.kv_append([self.key_cache[layer_idx]], [self.value_cache[layer_idx]], [key_states],
                                [value_states], self._zero_start)
        if layer_idx >= self._num_initialized:
            self._num_initialized = layer_idx + 1
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def write_at(self, key_states, value_states, layer_idx, start: torch.Tensor):
        """Sub-block write at `start` (device int32 [B]); the slice copy of
        attention_backends.py:862-866."""
        torch.ops.fdl.kv_append([self.key_cache[layer_idx]], [self.value_cache[layer_idx]], [key_states],
                                [value_states], start)

    def __getitem__(self, layer_idx):
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def __len__(self):
        return self._num_initialized

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return 0 if self._num_initialized == 0 else self.block_size

    def reset(self):
        self._num_initialized = 0

    def compact_batch(self, active_indices: torch.Tensor):
        """In place, like StaticKVCache.compact_batch (reference:
        utils/static_kv_cache.py:473-491)."""
        act = active_rows(active_indices, self.batch_size, self.device)
        n = act.numel()
        compact_rows(self.key_cache + self.value_cache, act)
        self.key_cache = [t[:n] for t in self.key_cache]
        self.value_cache = [t[:n] for t in self.value_cache]
        self._zero_start = self._zero_start[:n]
        self.batch_size = n
