"""CPU oracle for the token selection that feeds the sparse gathers -- TEST
INFRASTRUCTURE ONLY (tests, ``__graft_entry__.smoke()``, ``bench.py``'s CPU
legs).  Nothing in the product path imports it.

Restated here (reference paths relative to the reference repository root;
``modeling.py`` abbreviates
models/models--Efficient-Large-Model--Fast_dLLM_v2_7B/snapshots/0661abf5f9f0ee338970d091052a26c8efa51974/modeling.py):

* ``cosine_select``      the token selection of the sparse forward
                         (modeling.py:868-874): cosine similarity of each
                         block token's layer input with the cached one, the
                         ``n`` least similar tokens, sorted.
* ``focus_importance``   ``_focus_importance`` (modeling.py:214-237).
* ``focus_select``       ``_focus_select`` (modeling.py:240-306).

The reference runs these in the model dtype.  For bf16 inputs every step
rounds to bf16 where torch's bf16 op would (each elementwise op, each
reduction's output); fp32 inputs are not rounded.  ``torch.topk`` leaves the
order of equal values to the implementation; here, as in the CUDA kernels,
equal values are ranked by position (lower index first).

The two index functions must equal the CUDA kernels bit for bit on the same
inputs, so their float32 reductions follow the kernels' order exactly: a
warp's 32 lanes accumulate in a fixed element order and then combine with an
xor-shuffle butterfly (offsets 16, 8, 4, 2, 1).  The importance is floating
point and is compared with a tolerance.  tests/test_oracle_select_cpu.py pins
all three against the reference's own functions run on CPU
(tests/golden/make_golden.py, ``select.npz``) and restates the reference's
known-answer tests (tests/test_focus.py:32-124).
"""
from __future__ import annotations

import numpy as np

from .kvcache_oracle import bf16_to_f32, f32_to_bf16

F32 = np.float32
LANES = 32
BF16_MIN = -3.3895313892515355e38  # torch.finfo(torch.bfloat16).min
F32_MIN = float(np.finfo(np.float32).min)


def rnd(x, bf16: bool):
    """Round float32 values to bf16 (and back) in bf16 mode; identity otherwise."""
    x = np.asarray(x, dtype=F32)
    return bf16_to_f32(f32_to_bf16(x)) if bf16 else x


def butterfly_sum(v):
    """Sum over the last axis (the 32 lanes of a warp) in the order of an
    xor-shuffle reduction; every lane ends with the same float32 value."""
    v = np.asarray(v, dtype=F32)
    lanes = np.arange(LANES)
    for off in (16, 8, 4, 2, 1):
        v = (v + v[..., lanes ^ off]).astype(F32)
    return v[..., 0]


def lane_sum(terms, vec: int):
    """Row sums of ``terms`` [R, H] as one warp computes them: lane l adds the
    16-byte chunks l, l + 32, l + 64, ... (``vec`` elements each, in order)
    into one float32 accumulator, then the butterfly combines the lanes."""
    terms = np.asarray(terms, dtype=F32)
    R, H = terms.shape
    n_chunk = H // vec
    per_lane = -(-n_chunk // LANES)
    pad = np.zeros((R, per_lane * LANES * vec), dtype=F32)
    pad[:, :H] = terms
    # [R, t, lane, e]: element index = ((t * 32) + lane) * vec + e
    t4 = pad.reshape(R, per_lane, LANES, vec)
    acc = np.zeros((R, LANES), dtype=F32)
    for t in range(per_lane):
        for e in range(vec):
            acc = (acc + t4[:, t, :, e]).astype(F32)
    return butterfly_sum(acc)


def rank_select(values, n: int, largest: bool):
    """Boolean mask of the ``n`` largest (or smallest) entries of every row,
    equal values ranked by position (lower index first)."""
    v = np.asarray(values, dtype=np.float64)
    B, S = v.shape
    out = np.zeros((B, S), dtype=bool)
    idx = np.arange(S)
    for b in range(B):
        for i in range(S):
            better = (v[b] > v[b, i]) if largest else (v[b] < v[b, i])
            rank = int(np.sum(better | ((v[b] == v[b, i]) & (idx < i))))
            out[b, i] = rank < n
    return out


def sorted_indices(sel):
    """[B, n] ascending positions of a boolean selection with n per row."""
    return np.stack([np.nonzero(r)[0] for r in sel]).astype(np.int64)


# --------------------------------------------------------------------------
# cosine-similarity selection (modeling.py:868-874)
# --------------------------------------------------------------------------


def cosine_similarity_rows(x, y, bf16: bool, eps: float = 1e-8):
    """F.cosine_similarity(x, y, dim=-1) over [R, H] rows, as torch computes
    it: each input divided by its clamped L2 norm, the products summed
    (x / max(||x||, eps)) . (y / max(||y||, eps)); in bf16 every op's output
    is rounded to bf16.  Reductions in the kernel's lane order."""
    x = np.asarray(x, dtype=F32)
    y = np.asarray(y, dtype=F32)
    vec = 8 if bf16 else 4
    e = rnd(np.float32(eps), bf16).item()
    n1 = np.maximum(rnd(np.sqrt(lane_sum((x * x).astype(F32), vec)), bf16), F32(e))
    n2 = np.maximum(rnd(np.sqrt(lane_sum((y * y).astype(F32), vec)), bf16), F32(e))
    a = rnd((x / n1[:, None]).astype(F32), bf16)
    b = rnd((y / n2[:, None]).astype(F32), bf16)
    return rnd(lane_sum(rnd((a * b).astype(F32), bf16), vec), bf16)


def cosine_select(hidden, cached, n: int, bf16: bool):
    """The ``n`` block tokens whose layer input moved most (lowest cosine
    similarity with the cached input), ascending: modeling.py:868-874
    (``cos_sim.topk(n, largest=False).indices.sort()``).  hidden / cached:
    float32 [B, S, H] (bf16-representable in bf16 mode).  Returns
    (indices [B, n] int64, cos [B, S] float32)."""
    B, S, H = hidden.shape
    cos = cosine_similarity_rows(hidden.reshape(B * S, H), cached.reshape(B * S, H), bf16).reshape(B, S)
    return sorted_indices(rank_select(cos, n, largest=False)), cos


# --------------------------------------------------------------------------
# FOCUS importance (modeling.py:214-237)
# --------------------------------------------------------------------------


def focus_importance(q, k, mask_idx, scaling: float, bf16: bool):
    """Attention mass each masked key receives from masked queries, summed
    over heads.  q [B, Hq, S, D], k [B, Hkv, S, D] (Hkv divides Hq: query
    head h reads key head h // (Hq / Hkv), as repeat_kv); mask_idx [B, S].
    Scores rounded like torch's matmul output, then times the scale, masked,
    max-pooled over 3 neighbouring keys, masked again, softmaxed, zeroed for
    fully masked rows and for unmasked queries, summed over queries (one
    rounding) and over heads (one rounding).  float64 arithmetic between the
    rounding points; returns float32 [B, S]."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    m = np.asarray(mask_idx, dtype=bool)
    B, Hq, S, D = q.shape
    rep = Hq // k.shape[1]

    def r(x):
        return rnd(np.asarray(x, dtype=np.float64).astype(F32), bf16).astype(np.float64)

    sc = float(np.float32(scaling))  # the Python float scale, as fp32 opmath
    per_head = np.zeros((B, Hq, S))
    for h in range(Hq):
        s = r(np.einsum("bid,bjd->bij", q[:, h], k[:, h // rep]))
        s = r(s * sc)
        s = np.where(m[:, None, :], s, -np.inf)
        left = np.concatenate([np.full((B, S, 1), -np.inf), s[:, :, :-1]], axis=2)
        right = np.concatenate([s[:, :, 1:], np.full((B, S, 1), -np.inf)], axis=2)
        p = np.maximum(np.maximum(left, s), right)
        p = np.where(m[:, None, :], p, -np.inf)
        mx = p.max(axis=2, keepdims=True)
        with np.errstate(invalid="ignore"):
            e = np.exp(p - mx)
            w = r(e / e.sum(axis=2, keepdims=True))
        w = np.nan_to_num(w, nan=0.0)
        w = w * m[:, :, None]
        per_head[:, h] = r(w.sum(axis=1))
    return r(per_head.sum(axis=1)).astype(F32)


# --------------------------------------------------------------------------
# FOCUS selection (modeling.py:240-306)
# --------------------------------------------------------------------------


def focus_retain_k(S: int, avg_decoded: float, focus_alpha: float, retain_override=None) -> int:
    """The retain target K of _focus_select (modeling.py:254-257), host math."""
    import math

    if retain_override is not None:
        return max(1, min(S, int(math.ceil(retain_override * S))))
    return max(1, min(S, int(math.ceil(avg_decoded * focus_alpha))))


def focus_select(delta, mask_idx, K: int, bf16: bool, frozen=None):
    """_focus_select (modeling.py:240-306) for one block.  delta float32
    [B, S] (bf16-representable in bf16 mode), mask_idx / frozen bool [B, S],
    K from ``focus_retain_k``.  Row statistics are reduced in the kernel's
    butterfly order.  Returns (token_indices [B, Ksel] int64 ascending, Ksel)."""
    d = np.asarray(delta, dtype=F32)
    valid = np.asarray(mask_idx, dtype=bool)
    B, S = d.shape
    neg = F32(BF16_MIN if bf16 else F32_MIN)

    def lanes(x):  # [B, S] -> [B, 32] lane values, zero-padded
        out = np.zeros((B, LANES), dtype=F32)
        out[:, :S] = x
        return out

    cnt = np.maximum(valid.sum(axis=1), 1).astype(F32)
    s1 = rnd(butterfly_sum(lanes(np.where(valid, d, F32(0)))), bf16)
    mean = rnd((s1 / cnt).astype(F32), bf16)
    dev = rnd((d - mean[:, None]).astype(F32), bf16)
    sq = rnd((dev * dev).astype(F32), bf16)
    s2 = rnd(butterfly_sum(lanes(np.where(valid, sq, F32(0)))), bf16)
    var = rnd((s2 / cnt).astype(F32), bf16)
    thr = rnd((mean + rnd(np.sqrt(var), bf16)).astype(F32), bf16)
    cand = valid & (d >= thr[:, None])
    adj = np.zeros_like(cand)
    adj[:, :-1] = cand[:, 1:]
    mustkeep = (cand | adj) & valid
    masked_delta = np.where(valid, d, neg)
    topk = rank_select(masked_delta, K, largest=True) & valid
    retain = (~valid) | ((mustkeep | topk) & valid)
    if frozen is not None:
        fz = np.asarray(frozen, dtype=bool)
        retain &= ~fz
    ksel = int(min(max(int(retain.sum(axis=1).max()), K), S))
    if frozen is not None:
        n_free = int((~fz).sum(axis=1).max())
        ksel = max(1, min(ksel, n_free))
    prio = np.where(retain, rnd((d + F32(1e4)).astype(F32), bf16), d)
    if frozen is not None:
        prio = np.where(fz, neg, prio)
    return sorted_indices(rank_select(prio, ksel, largest=True)), ksel
