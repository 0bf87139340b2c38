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


def rmsnorm(x, w, eps):
    """Fast_dLLM_QwenRMSNorm.forward (modeling.py:427-432)."""
    dt = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    return w * (h * torch.rsqrt(var + eps)).to(dt)


def swiglu(gu):
    """The activation of Fast_dLLM_QwenMLP.forward (modeling.py:163-165) on the
    fused gate/up projection output [.., 2F]: act_fn(gate) * up with act_fn =
    silu (Qwen2 hidden_act), in the tensor's dtype."""
    f = gu.shape[-1] // 2
    return F.silu(gu[..., :f]) * gu[..., f:]


def rope(x_bhsd, cos, sin):
    """apply_rotary_pos_emb (modeling.py:186-199), BHSD with cos/sin [1, S, D]."""
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    h = x_bhsd.shape[-1] // 2
    rot = torch.cat((-x_bhsd[..., h:], x_bhsd[..., :h]), dim=-1)
    return x_bhsd * cos + rot * sin


def dkv_full_step_forward(layers, embed, norm_w, lm_head, ids, prefix_k, prefix_v, past_len, geo):
    """One full dKV diffusion step of the reference (forward_dkv with
    is_full_step=True, modeling.py:1625-1662, through Fast_dLLM_QwenDecoderLayer
    and Fast_dLLM_QwenAttention.forward with dkv_store, modeling.py:327-415):
    embed -> per layer [RMSNorm, q/k/v, RoPE, cat(prefix, block), repeat_kv +
    SDPA under eval_mask, o_proj, residual, RMSNorm, SwiGLU MLP, residual] ->
    norm -> lm_head.  `layers` holds per-layer dicts of torch weights
    (wq, bq, wk, bk, wv, bv, wo, ln1, ln2, wg, wu, wd); prefix_k/v are
    per-layer BHSD [B, Hkv, P, D].  Runs on the device of `ids` (CPU for the
    timed baseline, the GPU for the agreement test at full geometry)."""
    B, T = ids.shape
    D, Hq, Hkv = geo["head_dim"], geo["heads"], geo["kv_heads"]
    dev = ids.device
    h = F.embedding(ids, embed)
    pos = torch.arange(past_len, past_len + T, dtype=torch.float32, device=dev)
    inv = 1.0 / (geo["rope_theta"] ** (torch.arange(0, D, 2, dtype=torch.int64, device=dev).float() / D))
    f = pos[:, None] * inv[None, :]
    emb = torch.cat((f, f), dim=-1)
    cos, sin = emb.cos().to(h.dtype)[None], emb.sin().to(h.dtype)[None]
    qi = torch.arange(T, device=dev)[:, None] + past_len
    kj = torch.arange(T + prefix_k[0].shape[2], device=dev)[None, :]
    mask = (qi // 32) >= (kj // 32)
    for l, w in enumerate(layers):
        res = h
        x = rmsnorm(h, w["ln1"], geo["eps"])
        q = F.linear(x, w["wq"], w["bq"]).view(B, T, Hq, D).transpose(1, 2)
        k = F.linear(x, w["wk"], w["bk"]).view(B, T, Hkv, D).transpose(1, 2)
        v = F.linear(x, w["wv"], w["bv"]).view(B, T, Hkv, D).transpose(1, 2)
        q, k = rope(q, cos, sin), rope(k, cos, sin)
        fk = torch.cat((prefix_k[l], k), dim=-2)
        fv = torch.cat((prefix_v[l], v), dim=-2)
        n_rep = Hq // Hkv
        fk = fk[:, :, None].expand(-1, -1, n_rep, -1, -1).reshape(B, Hq, -1, D)
        fv = fv[:, :, None].expand(-1, -1, n_rep, -1, -1).reshape(B, Hq, -1, D)
        a = F.scaled_dot_product_attention(q, fk, fv, attn_mask=mask, scale=D ** -0.5)
        h = res + F.linear(a.transpose(1, 2).reshape(B, T, Hq * D), w["wo"])
        x = rmsnorm(h, w["ln2"], geo["eps"])
        h = h + F.linear(F.silu(F.linear(x, w["wg"])) * F.linear(x, w["wu"]), w["wd"])
    h = rmsnorm(h, norm_w, geo["eps"])
    return F.linear(h, lm_head)
