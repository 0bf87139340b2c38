"""Attention backend for Fast-dLLM v2 on B200 (drop-in for
utils/attention_backends.py).

The reference probes FA4 -> FA3 -> FA2 -> FlashInfer -> SDPA
(utils/attention_backends.py:685-770).  Here there is exactly one backend,
``fdl_b200``: the tcgen05/TMEM block-attention kernel of libfdl_b200.so with
GQA packed into the MMA tile.  ``get_attention_backend(preference)`` accepts
the reference's preference strings for compatibility and always returns it;
``plan_flashinfer`` is a no-op (the kernel needs no plan: per-sequence lengths
are read on the device).

``patch_attention_layers`` / ``patch_attention_layers_compiled`` /
``unpatch_attention_layers`` replace the model's attention forwards exactly as
the reference does (utils/attention_backends.py:791-1019); the cache writes
they issue go to the StaticKVCache kernels and the attention to
``flash_kvcache_attention`` below.
"""
from __future__ import annotations

import logging
from functools import lru_cache
from typing import Optional

import torch

from .. import _lib
from .static_kv_cache import StaticBlockCache, StaticKVCache  # noqa: F401

logger = logging.getLogger(__name__)


class AttentionBackend:
    """Single-backend form of the reference's AttentionBackend
    (utils/attention_backends.py:293-682)."""

    FDL = "fdl_b200"
    # Reference names kept so `attn_backend.name == "flashinfer"` style checks
    # in callers stay valid (they are simply false here).
    SDPA = "sdpa"
    FLASH2 = "flash2"
    FLASH3 = "flash3"
    FLASH4 = "flash4"
    FLASHINFER = "flashinfer"

    def __init__(self, name: str = FDL, impl=None):
        if name != self.FDL:
            raise ValueError(f"fast_v2_b200 provides only the {self.FDL!r} backend, not {name!r}")
        _lib.ensure_ops()
        self.name = name
        self._impl = impl
        self._kvcache_dispatch_logged = False
        self._ws = None

    def mark_dispatch_logged(self):
        self._kvcache_dispatch_logged = True

    def plan_flashinfer(self, *args, **kwargs):
        """No-op: the kernel reads per-sequence lengths on the device."""
        return None

    def attention(self, query, key, value, attn_mask: Optional[torch.Tensor] = None, scaling: float = None,
                  is_causal: bool = False, dropout: float = 0.0) -> torch.Tensor:
        """BHSD attention over all keys (utils/attention_backends.py:332-360);
        supports attn_mask=None, is_causal=False, dropout=0 (the inference
        configurations of the reference)."""
        if attn_mask is not None or is_causal or dropout:
            raise NotImplementedError("fdl_b200 attention(): only mask-free, non-causal, dropout-free attention")
        B, Hq, Sq, D = query.shape
        q = query.transpose(1, 2).contiguous()
        k = key.transpose(1, 2)
        v = value.transpose(1, 2)
        seq = torch.full((B,), key.shape[2], dtype=torch.int32, device=query.device)
        scale = scaling if scaling is not None else D ** -0.5
        return torch.ops.fdl.flash_kvcache(q, k, v, seq, float(scale), False).transpose(1, 2)

    def flash_kvcache_attention(self, query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                cache_seqlens: torch.Tensor, is_causal: bool = False,
                                scaling: float = None) -> torch.Tensor:
        """Attention of query [B, S_q, H, D] over the static KV buffers
        [B, max_S, H_kv, D] with valid keys j < cache_seqlens[b]
        (utils/attention_backends.py:588-640).  Returns BSHD."""
        scale = scaling if scaling is not None else query.shape[-1] ** -0.5
        if not self._kvcache_dispatch_logged and not torch.compiler.is_compiling():
            logger.info("[flash_kvcache_attention] backend=%r query=%s kv_cache=%s", self.name,
                        tuple(query.shape), tuple(k_cache.shape))
            self._kvcache_dispatch_logged = True
        if cache_seqlens.dtype != torch.int32:
            cache_seqlens = cache_seqlens.to(torch.int32)
        return torch.ops.fdl.flash_kvcache(query, k_cache, v_cache, cache_seqlens, float(scale), bool(is_causal))

    def block_attention(self, query, k_prefix, v_prefix, prefix_lens, k_block=None, v_block=None, out=None,
                        mask_block: int = 0, q_pos=None, scaling: float = None, workspace=None, num_splits: int = 0):
        """Attention over cat(prefix[:prefix_lens[b]], block) with the block
        appended logically (no concatenation in memory).  All tensors BSHD-
        strided; returns `out` (allocated when None)."""
        if out is None:
            out = torch.empty_like(query, memory_format=torch.contiguous_format)
        D = query.shape[-1]
        scale = scaling if scaling is not None else D ** -0.5
        if workspace is None and num_splits != 1:
            B, Sq, Hq, _ = query.shape
            nblk = k_block.shape[1] if k_block is not None else 0
            ns = num_splits or _lib.attn_auto_splits(B, Sq, Hq, k_prefix.shape[2], k_prefix.shape[1], nblk)
            wsb = _lib.attn_workspace_bytes(B, Sq, Hq, ns)
            if wsb > 0:
                workspace = torch.empty(wsb, dtype=torch.uint8, device=query.device)
            num_splits = ns
        torch.ops.fdl.block_attn(query, k_prefix, v_prefix, prefix_lens, k_block, v_block, q_pos, mask_block,
                                 float(scale), out, workspace, num_splits)
        return out


@lru_cache(maxsize=1)
def get_attention_backend(preference: str = "auto") -> AttentionBackend:
    """Return the B200 backend; the reference's preferences ("auto", "flash2",
    "flashinfer", "sdpa", ...) all resolve to it."""
    logger.info("[attention_backend] SELECTED: %s (requested=%r)", AttentionBackend.FDL, preference)
    return AttentionBackend(AttentionBackend.FDL, None)


def _apply_rotary_pos_emb(q, k, cos, sin):
    """RoPE on BSHD q/k (utils/attention_backends.py:777-788)."""
    cos = cos.unsqueeze(2)
    sin = sin.unsqueeze(2)
    half = q.shape[-1] // 2
    q_embed = (q * cos) + (torch.cat((-q[..., half:], q[..., :half]), dim=-1) * sin)
    k_embed = (k * cos) + (torch.cat((-k[..., half:], k[..., :half]), dim=-1) * sin)
    return q_embed, k_embed


def _create_patched_attention_forward(attn_module, attn_backend, static_block_cache=None):
    """Patched attention forward (utils/attention_backends.py:791-898)."""
    original_forward = attn_module.forward
    layer_idx = attn_module.layer_idx
    head_dim = attn_module.head_dim
    scaling = attn_module.scaling

    def patched_forward(hidden_states, position_embeddings, attention_mask=None, past_key_value=None,
                        cache_position=None, update_past_key_values=False, block_past_key_values=None,
                        replace_position=None, **kwargs):
        if not isinstance(past_key_value, StaticKVCache):
            return original_forward(hidden_states, position_embeddings, attention_mask, past_key_value,
                                    cache_position, update_past_key_values, block_past_key_values,
                                    replace_position, **kwargs)
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, head_dim)
        query_states = attn_module.q_proj(hidden_states).view(hidden_shape)
        key_states = attn_module.k_proj(hidden_states).view(hidden_shape)
        value_states = attn_module.v_proj(hidden_states).view(hidden_shape)
        cos, sin = position_embeddings
        query_states, key_states = _apply_rotary_pos_emb(query_states, key_states, cos, sin)
        if block_past_key_values is not None:
            if len(block_past_key_values) <= layer_idx:
                key_states, value_states = block_past_key_values.update(
                    key_states, value_states, layer_idx, {"sin": sin, "cos": cos, "cache_position": cache_position})
            else:
                bk, bv = block_past_key_values[layer_idx]
                seq_len = key_states.shape[1]
                rp = 0 if replace_position is None else replace_position
                bk[:, rp:rp + seq_len].copy_(key_states)
                bv[:, rp:rp + seq_len].copy_(value_states)
                key_states, value_states = bk, bv
        if update_past_key_values:
            past_len = past_key_value.get_seq_length()
            seq_len = key_states.shape[1]
            past_key_value.update(key_states, value_states, layer_idx)
            past_key_value.set_scratch_seqlens(past_len + seq_len)
        else:
            past_key_value.write_scratch_compiled(key_states, value_states, layer_idx)
        full_k, full_v = past_key_value.get_full_kv(layer_idx)
        attn_output = attn_backend.flash_kvcache_attention(query_states, full_k, full_v,
                                                           cache_seqlens=past_key_value.scratch_seqlens,
                                                           is_causal=False, scaling=scaling)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        return attn_module.o_proj(attn_output)

    return patched_forward


def _create_compiled_attention_forward(attn_module, attn_backend):
    """Branch-free forward for the compiled diffusion step
    (utils/attention_backends.py:901-974)."""
    layer_idx = attn_module.layer_idx
    head_dim = attn_module.head_dim
    scaling = attn_module.scaling

    def compiled_forward(hidden_states, position_embeddings, attention_mask=None, past_key_value=None,
                         cache_position=None, update_past_key_values=False, block_past_key_values=None,
                         replace_position=None, **kwargs):
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, head_dim)
        query_states = attn_module.q_proj(hidden_states).view(hidden_shape)
        key_states = attn_module.k_proj(hidden_states).view(hidden_shape)
        value_states = attn_module.v_proj(hidden_states).view(hidden_shape)
        cos, sin = position_embeddings
        query_states, key_states = _apply_rotary_pos_emb(query_states, key_states, cos, sin)
        past_key_value.write_scratch_compiled(key_states, value_states, layer_idx)
        full_k, full_v = past_key_value.get_full_kv(layer_idx)
        attn_output = attn_backend.flash_kvcache_attention(query_states, full_k, full_v,
                                                           cache_seqlens=past_key_value.scratch_seqlens,
                                                           is_causal=False, scaling=scaling)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        return attn_module.o_proj(attn_output)

    return compiled_forward


def patch_attention_layers(model, attn_backend, static_block_cache=None):
    original_forwards = {}
    for i, layer in enumerate(model.model.layers):
        attn = layer.self_attn
        original_forwards[i] = attn.forward
        attn.forward = _create_patched_attention_forward(attn, attn_backend, static_block_cache)
    return original_forwards


def patch_attention_layers_compiled(model, attn_backend):
    original_forwards = {}
    for i, layer in enumerate(model.model.layers):
        attn = layer.self_attn
        original_forwards[i] = attn.forward
        attn.forward = _create_compiled_attention_forward(attn, attn_backend)
    return original_forwards


def unpatch_attention_layers(model, original_forwards):
    for i, layer in enumerate(model.model.layers):
        if i in original_forwards:
            layer.self_attn.forward = original_forwards[i]
