"""Token selection of the sparse and FOCUS steps on the GPU.

Drop-ins for the module-level helpers of the reference's modeling.py
(``_focus_importance``, ``_focus_select``) and for the cosine top-k of its
sparse forward; a caller swaps them in by name, e.g.
``modeling._focus_select = fast_v2_b200.focus.focus_select``.  Each runs one
sm_100a kernel (``fdl_focus_importance``, ``fdl_focus_select``,
``fdl_cosine_select``); inputs stay on the device, and the only host read is
the batch-uniform selection width of ``focus_select``, which the reference
reads with ``.item()`` as well (modeling.py:286).

The selections are exact: float reductions run in a fixed order and bf16
inputs are rounded wherever the reference's bf16 torch ops round.
``torch.topk`` leaves the order of equal values open; here equal values rank
by position, lower index first.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib


def focus_importance(q: torch.Tensor, k: torch.Tensor, mask_idx: torch.Tensor, scaling: float) -> torch.Tensor:
    """_focus_importance (modeling.py:214-237): [B, S] attention mass each
    masked token receives from masked queries, max-pooled over 3 keys,
    softmaxed, summed over queries and heads.  q [B, H, S, d]; k [B, H, S, d]
    as the reference passes it (after repeat_kv) or [B, H_kv, S, d] without
    the copy -- query head h reads key head h // (H / H_kv)."""
    _lib.ensure_ops()
    B, _, S, _ = q.shape
    imp = torch.empty(B, S, dtype=q.dtype, device=q.device)
    torch.ops.fdl.focus_importance(q, k, mask_idx.to(torch.bool), float(scaling), imp)
    return imp


def focus_retain_k(S: int, avg_decoded: float, focus_alpha: float, retain_override: Optional[float] = None) -> int:
    """The retain target of _focus_select (modeling.py:254-257)."""
    if retain_override is not None:
        return max(1, min(S, int(math.ceil(retain_override * S))))
    return max(1, min(S, int(math.ceil(avg_decoded * focus_alpha))))


def focus_select(delta: torch.Tensor, mask_idx: torch.Tensor, avg_decoded: float, focus_alpha: float,
                 retain_override: Optional[float] = None, frozen: Optional[torch.Tensor] = None):
    """_focus_select (modeling.py:240-306): (token_indices [B, Ksel] int64
    ascending, Ksel).  Decoded tokens are retained, masked tokens above the
    mean + std threshold (and their left neighbours) and the top-K masked
    deltas are selected, frozen tokens are dropped; the width is padded with
    the highest-delta remaining tokens."""
    _lib.ensure_ops()
    B, S = delta.shape
    K = focus_retain_k(S, avg_decoded, focus_alpha, retain_override)
    sel = torch.empty(B, S, dtype=torch.long, device=delta.device)
    ksel = torch.empty(1, dtype=torch.int32, device=delta.device)
    torch.ops.fdl.focus_select(delta, mask_idx.to(torch.bool), None if frozen is None else frozen.to(torch.bool), K,
                               sel, ksel)
    n = int(ksel.item())
    return sel[:, :n], n


def cosine_select(hidden_states: torch.Tensor, cached_input: torch.Tensor, num_tokens: int,
                  refresh_cache: bool = False, cos_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The sparse forward's token choice (modeling.py:868-874): the
    ``num_tokens`` block tokens whose layer input has the lowest cosine
    similarity with the cached input, ascending [B, num_tokens] int64.  With
    ``refresh_cache`` the cached input is overwritten with ``hidden_states``
    in the same pass (BlockSparseCache.cache_layer_input, modeling.py:877)."""
    _lib.ensure_ops()
    B = hidden_states.shape[0]
    idx = torch.empty(B, num_tokens, dtype=torch.long, device=hidden_states.device)
    torch.ops.fdl.cosine_select(hidden_states, cached_input, int(num_tokens), bool(refresh_cache), idx, cos_out)
    return idx
