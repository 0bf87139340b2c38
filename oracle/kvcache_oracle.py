"""CPU oracle for the Fast-dLLM v2 KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what the reference (navneet-13/fast_v2) computes
on the path the CUDA library accelerates.  It is the checker for the parity
tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py``; nothing in the product path imports it.

Pinning: every function is checked (tests/test_oracle_golden.py) against
golden vectors produced by running the reference's own Python code on CPU
(tests/golden/make_golden.py, fixtures in tests/golden/*.npz) and against the
reference's known-answer tests (tests/test_dkv.py, tests/test_focus.py of the
reference, restated in tests/test_oracle_known_answers.py).  The token-sparse
prefix selection (``sparse_prefix_select``) has no counterpart in the
reference: its specification is the docstring below and its parity is
unpinned by construction.

Arrays: bf16 data is carried as numpy ``uint16`` bit patterns (``bf16_bits``)
so copies are compared bit for bit; arithmetic converts to float32 exactly.
Reference paths below are relative to the reference repository root;
``modeling.py`` abbreviates
models/models--Efficient-Large-Model--Fast_dLLM_v2_7B/snapshots/0661abf5f9f0ee338970d091052a26c8efa51974/modeling.py.
"""
from __future__ import annotations

import math

import numpy as np

# --------------------------------------------------------------------------
# bf16 helpers (bit-exact conversions; round-to-nearest-even)
# --------------------------------------------------------------------------


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even, NaN kept quiet) -> uint16 bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


# --------------------------------------------------------------------------
# (a) KV append / scatter
# --------------------------------------------------------------------------


def kv_update_uniform(k_cache, v_cache, k, v, start: int):
    """StaticKVCache.update: slice copy of [B, S, H, D] at one start for the whole
    batch (utils/static_kv_cache.py:132-160).  In place; returns the caches."""
    s = k.shape[1]
    k_cache[:, start:start + s] = k
    v_cache[:, start:start + s] = v
    return k_cache, v_cache


def kv_append(k_cache, v_cache, k, v, start_pos):
    """Per-sequence append: row b lands at start_pos[b] .. start_pos[b]+S-1.
    With every start_pos[b] equal this is StaticKVCache.update
    (utils/static_kv_cache.py:147-152) / write_scratch_compiled with
    kv_write_start (utils/static_kv_cache.py:201-229); with per-row starts it is
    write_sparse at positions start_pos[:, None] + arange(S)
    (utils/static_kv_cache.py:231-247)."""
    s = k.shape[1]
    for b in range(k.shape[0]):
        p = int(start_pos[b])
        k_cache[b, p:p + s] = k[b]
        v_cache[b, p:p + s] = v[b]
    return k_cache, v_cache


def scatter_rows(dst, src, positions, seq_axis: int = 1):
    """dst[b, pos[b, i]] (along seq_axis) = src[b, i], applied in increasing i, so a
    repeated position keeps the LAST write -- torch.Tensor.scatter_ on CPU, as
    used by StaticKVCache.write_sparse (utils/static_kv_cache.py:231-247),
    DynamicBlockKV.write (utils/dynamic_block_kv.py:39-43, seq_axis=2) and
    BlockSparseCache.scatter_* (utils/block_sparse_cache.py:112-132)."""
    B, n = positions.shape
    for b in range(B):
        for i in range(n):
            p = int(positions[b, i])
            if seq_axis == 1:
                dst[b, p] = src[b, i]
            else:
                dst[b, :, p] = src[b, :, i]
    return dst


# --------------------------------------------------------------------------
# (b) prefix gathers
# --------------------------------------------------------------------------


def repeat_kv_bshd(x, n_rep: int):
    """repeat_kv (modeling.py:202-211) on the BSHD layout: head h of the output
    is head h // n_rep of the input."""
    return np.repeat(x, n_rep, axis=2)


def gather_prefix_packed(cache, lens, rep: int = 1, block=None):
    """Varlen prefix gather: concat over b of cache[b, :lens[b]] (+ block[b]) with
    GQA expansion, packed as [sum_b L_b, H*rep, D] plus cu_seqlens.  This is the
    slicing of StaticKVCache.get_kv_up_to (utils/static_kv_cache.py:279-284),
    torch.cat(prefix, block) of the dynamic path (modeling.py:390-392) and
    repeat_kv (modeling.py:202-211)."""
    parts, cu = [], [0]
    for b in range(cache.shape[0]):
        seg = cache[b, : int(lens[b])]
        if block is not None:
            seg = np.concatenate([seg, block[b]], axis=0)
        parts.append(np.repeat(seg, rep, axis=1))
        cu.append(cu[-1] + seg.shape[0])
    return np.concatenate(parts, axis=0), np.asarray(cu, dtype=np.int32)


def concat_bhsd(prefix, block):
    """torch.cat((past_k, k_block), dim=-2) on BHSD tensors (modeling.py:390-392)."""
    return np.concatenate([prefix, block], axis=2)


def gather_rows(src, idx, seq_axis: int = 1):
    """src.gather along the sequence axis with per-row indices
    (modeling.py:1232-1238, :1590-1592, :1661-1663)."""
    B = idx.shape[0]
    if seq_axis == 1:
        return np.stack([src[b, idx[b]] for b in range(B)])
    return np.stack([src[b][:, idx[b]] for b in range(B)])


def batch_compact(buf, active, batch_axis: int = 0):
    """``t[active_indices].contiguous()`` along the batch axis: the reference's
    compaction of every batch-indexed cache buffer
    (utils/static_kv_cache.py:366-379, :483-490; utils/dynamic_block_kv.py:52-56;
    utils/block_sparse_cache.py:143-146 with the batch on axis 1)."""
    return np.take(buf, np.asarray(active, dtype=np.int64), axis=batch_axis)


def batch_compact_in_place(buf, active):
    """The in-place order of the CUDA compaction, restated sequentially: for
    i = 0, 1, ... row i takes row active[i] of the partly updated buffer.
    Equal to ``batch_compact`` on the first len(active) rows whenever
    i <= active[i] < batch for every i; returns False (buffer untouched)
    for any other list, as the kernel reports it and moves nothing."""
    active = np.asarray(active, dtype=np.int64)
    n = active.shape[0]
    if np.any(active < np.arange(n)) or np.any(active >= buf.shape[0]):
        return False
    for i in range(n):
        if active[i] != i:
            buf[i] = buf[active[i]]
    return True


def key_norm_scores(k_bits, lens):
    """Token-sparse prefix score (no reference counterpart; specification):
    score[b, t] = sqrt(sum over (h, d) of K[b, t, h, d]^2) in fp32 for t < lens[b],
    with the summation order fixed so CPU and GPU agree bit for bit:
    the H*D elements of a token, in memory order, are split into 8-element
    vectors; vector v belongs to lane v % 32; each lane sums its vectors' squares
    sequentially in fp32 (vector by vector, element by element), then the 32
    lane sums are reduced by an xor butterfly with offsets 16, 8, 4, 2, 1
    (lane sum + partner sum, fp32).  Squares of bf16 values are exact in fp32.
    Returns fp32 [B, cap]; entries t >= lens[b] are 0."""
    B, cap = k_bits.shape[:2]
    e = int(np.prod(k_bits.shape[2:]))
    assert e % 8 == 0
    nvec = e // 8
    x = bf16_to_f32(k_bits.reshape(B, cap, nvec, 8))
    acc = np.zeros((B, cap, 32), dtype=np.float32)
    for lane_vec0 in range(0, nvec, 32):
        for lane in range(32):
            vi = lane_vec0 + lane
            if vi >= nvec:
                continue
            for j in range(8):
                xv = x[:, :, vi, j]
                acc[:, :, lane] = (acc[:, :, lane] + xv * xv).astype(np.float32)
    for off in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, :, np.arange(32) ^ off]).astype(np.float32)
    score = np.sqrt(acc[:, :, 0]).astype(np.float32)
    t = np.arange(cap)[None, :]
    score[t >= np.asarray(lens)[:, None]] = 0.0
    return score


def sparse_prefix_select(k_bits, lens, keep_num: int = 1, keep_den: int = 4, max_keep: int | None = None):
    """Token-sparse prefix selection (specification; parity unpinned):
    keep[b] = ceil(lens[b] * keep_num / keep_den); choose the keep[b] tokens of
    largest key_norm_scores, ties broken toward the lower index, and list them
    in ascending order.  Returns (sel int32 [B, max_keep] padded with -1,
    keep int32 [B])."""
    score = key_norm_scores(k_bits, lens)
    B = k_bits.shape[0]
    keeps = [-(-int(lens[b]) * keep_num // keep_den) for b in range(B)]
    mk = max(keeps + [1]) if max_keep is None else max_keep
    sel = np.full((B, mk), -1, dtype=np.int32)
    for b in range(B):
        L = int(lens[b])
        order = sorted(range(L), key=lambda t: (-float(score[b, t]), t))[: keeps[b]]
        order.sort()
        sel[b, : len(order)] = order
    return sel, np.asarray(keeps, dtype=np.int32)


# --------------------------------------------------------------------------
# (c) gather + RMSNorm
# --------------------------------------------------------------------------


def gather_rmsnorm_bf16(x_bits, idx, w_bits, eps: float):
    """ref_gather_input_rmsnorm (cuda_bench/test_correctness.py:33-50) ==
    Fast_dLLM_QwenRMSNorm.forward (modeling.py:427-432) on gathered rows:
    fp32 mean of squares, n = round_bf16(x * rsqrt(var + eps)),
    out = round_bf16(w * n).  Returns (gathered bits, normed bits)."""
    g = np.stack([x_bits[b, idx[b]] for b in range(x_bits.shape[0])])
    xf = bf16_to_f32(g).astype(np.float64)
    var = np.mean(xf * xf, axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(var + eps)).astype(np.float32)
    n = f32_to_bf16((bf16_to_f32(g) * inv).astype(np.float32))
    if w_bits is None:
        return g, n
    out = f32_to_bf16(bf16_to_f32(w_bits)[None, None, :] * bf16_to_f32(n))
    return g, out


def add_rmsnorm_bf16(x_bits, res_bits, w_bits, eps: float):
    """Decoder-layer residual connection followed by RMSNorm: the layer's
    `hidden_states = residual + hidden_states` (bf16 + bf16 -> one rounding)
    and then Fast_dLLM_QwenRMSNorm.forward (modeling.py:427-432) on the sum.
    Rows are the leading axes.  Returns (sum bits, normed bits)."""
    sm = f32_to_bf16((bf16_to_f32(x_bits) + bf16_to_f32(res_bits)).astype(np.float32))
    flat = sm.reshape(1, -1, sm.shape[-1])
    idx = np.arange(flat.shape[1])[None, :]
    _, n = gather_rmsnorm_bf16(flat, idx, w_bits, eps)
    return sm, n.reshape(sm.shape)


def gather_rmsnorm_f32(x, idx, w, eps: float):
    """select_gather_rmsnorm_kernel (cuda_bench/fused_gather_norm.cu:123-175):
    fp32 in/out, out = x * rsqrt(mean(x^2) + eps) (* w when given)."""
    g = np.stack([x[b, idx[b]] for b in range(x.shape[0])]).astype(np.float32)
    var = np.mean(g.astype(np.float64) ** 2, axis=-1, keepdims=True)
    n = (g * (1.0 / np.sqrt(var + eps))).astype(np.float32)
    if w is not None:
        n = (n * w[None, None, :]).astype(np.float32)
    return g, n


# --------------------------------------------------------------------------
# (d) block attention
# --------------------------------------------------------------------------


def block_attention(q, k, v, seqlens, scale=None, k_blk=None, v_blk=None, mask_block: int = 0, q_pos=None):
    """flash_kvcache_attention semantics (utils/attention_backends.py:588-640),
    restated as the SDPA stand-in of the reference tests
    (tests/test_focus.py:206-239): non-causal attention of q [B, Sq, Hq, D]
    over k/v [B, cap, Hkv, D] with keys j < seqlens[b] valid, GQA head
    h -> h // (Hq/Hkv) (modeling.py:202-211), softmax in float64 here.
    Optional block source appended after the first seqlens[b] keys
    (cat(prefix, block), modeling.py:390-392) and the block-causal mask
    qpos // mask_block >= kpos // mask_block (modeling.py:145-150, 585-593).
    A query with no visible key returns zeros.  Inputs are float arrays
    (already widened from bf16); returns float64 [B, Sq, Hq, D]."""
    B, Sq, Hq, D = q.shape
    Hkv = k.shape[2]
    G = Hq // Hkv
    scale = D ** -0.5 if scale is None else scale
    out = np.zeros((B, Sq, Hq, D), dtype=np.float64)
    for b in range(B):
        L = int(seqlens[b])
        kk = k[b, :L].astype(np.float64)
        vv = v[b, :L].astype(np.float64)
        kpos = np.arange(L)
        if k_blk is not None:
            kk = np.concatenate([kk, k_blk[b].astype(np.float64)], axis=0)
            vv = np.concatenate([vv, v_blk[b].astype(np.float64)], axis=0)
            kpos = np.concatenate([kpos, L + np.arange(k_blk.shape[1])])
        if kk.shape[0] == 0:
            continue
        for h in range(Hq):
            g = h // G
            s = (q[b, :, h].astype(np.float64) @ kk[:, g].T) * scale  # [Sq, n]
            if mask_block > 0:
                qp = (np.asarray(q_pos[b]) if q_pos is not None else L + np.arange(Sq))
                allowed = (qp[:, None] // mask_block) >= (kpos[None, :] // mask_block)
                s = np.where(allowed, s, -np.inf)
            mx = s.max(axis=1, keepdims=True)
            ok = np.isfinite(mx[:, 0])
            p = np.where(np.isfinite(s), np.exp(s - np.where(ok[:, None], mx, 0.0)), 0.0)
            den = p.sum(axis=1, keepdims=True)
            o = (p @ vv[:, g]) / np.where(den > 0, den, 1.0)
            o[~ok] = 0.0
            out[b, :, h] = o
    return out


def eval_block_mask(seqlen: int, block_size: int, cache_len: int):
    """Fast_dLLM_QwenModel.eval_mask (modeling.py:585-593) using
    eval_block_diff_mask (modeling.py:145-150): bool [seqlen, cache_len+seqlen],
    query i (absolute cache_len + i) sees key j iff (cache_len+i)//bs >= j//bs."""
    qi = np.arange(seqlen)[:, None] + cache_len
    kj = np.arange(seqlen + cache_len)[None, :]
    return (qi // block_size) >= (kj // block_size)


# --------------------------------------------------------------------------
# decode-forward elementwise stages next to the KV path
# --------------------------------------------------------------------------


def rope_qkv(y_bits, pos, inv_freq, hq: int, hkv: int):
    """q/k/v split of the fused projection output and rotary embedding:
    angle = fp32(pos * inv_freq) (Fast_dLLM_QwenRotaryEmbedding,
    modeling.py:545-560), c, s = bf16(cos/sin(angle)), and per element
    bf16(bf16(x * c) + bf16(rotate_half(x) * s)) (apply_rotary_pos_emb,
    modeling.py:186-199).  y_bits bf16 [rows, (hq + 2 hkv) * D] -> bits of
    q [rows, hq, D], k [rows, hkv, D], v [rows, hkv, D]."""
    rows = y_bits.shape[0]
    D = 2 * inv_freq.shape[0]
    y = bf16_to_f32(y_bits).reshape(rows, hq + 2 * hkv, D)
    ang = (np.asarray(pos, np.float32)[:, None] * inv_freq.astype(np.float32)[None, :]).astype(np.float32)
    c = bf16_to_f32(f32_to_bf16(np.cos(ang.astype(np.float64)).astype(np.float32)))
    s = bf16_to_f32(f32_to_bf16(np.sin(ang.astype(np.float64)).astype(np.float32)))
    c = np.concatenate([c, c], axis=1)[:, None, :]
    s = np.concatenate([s, s], axis=1)[:, None, :]

    def rnd(x):
        return bf16_to_f32(f32_to_bf16(x.astype(np.float32)))

    x = y[:, : hq + hkv]
    h = D // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    out = f32_to_bf16((rnd(x * c) + rnd(rot * s)).astype(np.float32))
    v = f32_to_bf16(y[:, hq + hkv:])
    return out[:, :hq], out[:, hq:], v


def swiglu(gu_bits):
    """bf16(bf16(silu(gate)) * up) over [rows, 2F] (Fast_dLLM_QwenMLP.forward,
    modeling.py:163-165: act_fn(gate_proj(x)) * up_proj(x) in bf16)."""
    F_ = gu_bits.shape[1] // 2
    g = bf16_to_f32(gu_bits[:, :F_]).astype(np.float64)
    u = bf16_to_f32(gu_bits[:, F_:])
    s = bf16_to_f32(f32_to_bf16((g / (1.0 + np.exp(-g))).astype(np.float32)))
    return f32_to_bf16((s * u).astype(np.float32))


# --------------------------------------------------------------------------
# index selection helpers on the path (a18)
# --------------------------------------------------------------------------


def dkv_fed_indices(prv_transfer_idx):
    """Fast_dLLM_QwenForCausalLM._dkv_fed_indices (modeling.py:2039-2060):
    fed = not-yet-frozen positions in ascending order, width = batch max
    count (>= 1), short rows padded with their first fed index."""
    fed = ~np.asarray(prv_transfer_idx, dtype=bool)
    counts = fed.sum(axis=1)
    num_fed = max(1, int(counts.max()))
    B, S = fed.shape
    out = np.zeros((B, num_fed), dtype=np.int64)
    for b in range(B):
        order = [i for i in range(S) if fed[b, i]] + [i for i in range(S) if not fed[b, i]]
        row = order[:num_fed]
        c = max(1, int(counts[b]))
        for j in range(num_fed):
            out[b, j] = row[j] if j < c else row[0]
    return out, num_fed


def focus_update_frozen(frozen, mask_idx):
    """_focus_update_frozen (modeling.py:2062-2080): freeze a decoded position
    whose right neighbour is decoded; OR-accumulating."""
    dec = ~np.asarray(mask_idx, dtype=bool)
    right = np.zeros_like(dec)
    right[:, :-1] = dec[:, 1:]
    return np.asarray(frozen, dtype=bool) | (dec & right)


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math", "np")]


# --------------------------------------------------------------------------
# greedy sampling statistics
# --------------------------------------------------------------------------


def softmax_argmax_bf16(logit_bits):
    """sample_with_top_p at temperature 0 (modeling.py:2263-2269) and the
    gathered probability of its token (generation_functions.py:2290-2291) on
    bf16 logits [rows, V] (uint16 bit patterns): probabilities
    bf16(exp(l - m) / s) with m the row max and s = sum exp(l - m) (float64
    here), token = the first index of the largest probability (argmax's
    first-occurrence rule), prob = that probability.  Returns (token int64
    [rows], prob bf16 bits [rows])."""
    x = bf16_to_f32(np.ascontiguousarray(logit_bits)).astype(np.float64)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    s = e.sum(axis=-1, keepdims=True)
    p = f32_to_bf16((e / s).astype(np.float32))
    pf = bf16_to_f32(p)
    tok = pf.argmax(axis=-1).astype(np.int64)
    return tok, np.take_along_axis(p, tok[:, None], axis=-1)[:, 0]
