"""The reference's torch code path for the KV-cache hot path, restated for CPU
timing -- TEST / BASELINE INFRASTRUCTURE ONLY.

``bench.py --impl reference`` and the ``cpu_baseline`` field time these
functions on the host cores (the reference repository itself does not travel to
the GPU box).  Each function performs the same torch operations, in the same
order, as the reference code it cites, so its CPU time is the reference's CPU
time for that work.  The product path never imports this module.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def gather_input_rmsnorm(hidden, token_indices, weight, eps):
    """cuda_bench/test_correctness.py:33-50 (ref_gather_input_rmsnorm), the torch
    path that cuda_bench/fused_gather_norm.cu replaces."""
    h = hidden.float().contiguous()
    b, _, dim = h.shape
    t = token_indices.shape[1]
    idx = token_indices.unsqueeze(-1).expand(b, t, dim)
    gathered_f = h.gather(1, idx)
    var = (gathered_f * gathered_f).mean(dim=-1, keepdim=True)
    inv = torch.rsqrt(var + eps)
    normed_pre = gathered_f * inv
    dt = hidden.dtype
    return gathered_f.to(dt), weight * normed_pre.to(dt)


def write_sparse(k_layer, v_layer, key_states, value_states, write_positions):
    """StaticKVCache.write_sparse (utils/static_kv_cache.py:231-247)."""
    idx = write_positions.unsqueeze(-1).unsqueeze(-1).expand(-1, -1, k_layer.shape[2], k_layer.shape[3])
    k_layer.scatter_(1, idx, key_states)
    v_layer.scatter_(1, idx, value_states)


def repeat_kv_bshd(x, n_rep):
    """repeat_kv (modeling.py:202-211) on a [S, H, D] prefix slice."""
    s, h, d = x.shape
    return x[:, :, None, :].expand(s, h, n_rep, d).reshape(s, h * n_rep, d)


def append_and_gather(k_caches, v_caches, k_new, v_new, lens, n_rep, layers):
    """One config-2 step on `layers`: per-sequence append of the block at
    lens[b] (write_sparse with positions lens[:, None] + arange) and the varlen
    prefix gather + GQA expansion (get_kv_up_to slicing, utils/static_kv_cache.py:
    279-284, + repeat_kv) packed over the batch."""
    B, n = k_new.shape[0], k_new.shape[1]
    pos = lens.to(torch.int64)[:, None] + torch.arange(n)[None, :]
    outs = []
    for l in layers:
        write_sparse(k_caches[l], v_caches[l], k_new, v_new, pos)
        ks, vs = [], []
        for b in range(B):
            L = int(lens[b]) + n
            ks.append(repeat_kv_bshd(k_caches[l][b, :L], n_rep))
            vs.append(repeat_kv_bshd(v_caches[l][b, :L], n_rep))
        outs.append((torch.cat(ks), torch.cat(vs)))
    return outs


def flash_kvcache_sdpa(query, k_cache, v_cache, cache_seqlens, scaling=None):
    """The SDPA form of flash_kvcache_attention used by the reference's tests
    (tests/test_focus.py:206-239): GQA expand, seqused -inf mask, SDPA."""
    B_, S_q, H_, D_ = query.shape
    max_S, H_kv = k_cache.shape[1], k_cache.shape[2]
    scale = scaling if scaling is not None else D_ ** -0.5
    q = query.transpose(1, 2)
    k = k_cache.transpose(1, 2)
    v = v_cache.transpose(1, 2)
    if H_ != H_kv:
        n_rep = H_ // H_kv
        k = k[:, :, None].expand(-1, -1, n_rep, -1, -1).reshape(B_, H_, max_S, D_)
        v = v[:, :, None].expand(-1, -1, n_rep, -1, -1).reshape(B_, H_, max_S, D_)
    pos = torch.arange(max_S)
    valid = pos[None, :] < cache_seqlens.to(torch.long)[:, None]
    attn_mask = torch.zeros(B_, 1, 1, max_S, dtype=q.dtype)
    attn_mask.masked_fill_(~valid[:, None, None, :], float("-inf"))
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, scale=scale)
    return out.transpose(1, 2).contiguous()
