"""Fused index-gather + RMSNorm for the token-sparse forward (drop-in for
cuda_bench/fused_sparse_extension.py of the reference).

Same public names and contracts as the reference module
(cuda_bench/fused_sparse_extension.py:25-87):

* ``get_fused_ops()`` returns an object exposing the four functions of the
  reference's pybind module (cuda_bench/fused_gather_norm.cu:215-221):
  ``gather_rmsnorm_cuda``, ``scatter_and_return_cuda``, ``fused_select_norm``,
  ``fused_gather_input_rmsnorm_pair``.  They run the sm_100a kernels of
  ``libfdl_b200.so`` (no JIT build).  Unlike the reference, a missing native
  library raises ``ImportError`` instead of returning ``None``: there is no
  silent fallback.
* ``fused_gather_input_rmsnorm_pair(hidden_states, token_indices, input_layernorm)``
  returns ``(gathered, normed)`` in the dtype of ``hidden_states``, with
  ``normed = weight * (x * rsqrt(mean(x^2) + eps)).to(dtype)`` exactly as
  Fast_dLLM_QwenRMSNorm.forward (modeling.py:427-432); ``None`` for non-CUDA
  input (reference contract, cuda_bench/fused_sparse_extension.py:66-67).
  The bf16 path reads the hidden rows once in bf16 -- the reference upcasts
  the whole hidden tensor to fp32 first (cuda_bench/fused_sparse_extension.py:82).
"""
from __future__ import annotations

from types import SimpleNamespace
from typing import Any, Optional, Tuple

import torch

from .. import _lib

_OPS: Any = None


def _out(like: torch.Tensor, b: int, t: int, h: int) -> torch.Tensor:
    return torch.empty(b, t, h, dtype=like.dtype, device=like.device)


def gather_rmsnorm_cuda(input: torch.Tensor, indices: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """out[b, t] = x[b, idx[b, t]] * rsqrt(mean(x^2) + eps) * weight (fused_gather_norm.cu:21-73)."""
    b, _, h = input.shape
    out = _out(input, b, indices.shape[1], h)
    torch.ops.fdl.gather_rmsnorm(input, indices.long(), weight.to(input.dtype).contiguous(), float(eps), None, out)
    return out


def fused_select_norm(hidden: torch.Tensor, indices: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Same computation as gather_rmsnorm_cuda (fused_gather_norm.cu:177-190)."""
    return gather_rmsnorm_cuda(hidden, indices, weight, eps)


def fused_gather_input_rmsnorm_pair_raw(hidden: torch.Tensor, indices: torch.Tensor, eps: float):
    """[gathered, x * rsqrt(mean(x^2) + eps)] without weight (fused_gather_norm.cu:193-209)."""
    b, _, h = hidden.shape
    t = indices.shape[1]
    gathered, normed = _out(hidden, b, t, h), _out(hidden, b, t, h)
    torch.ops.fdl.gather_rmsnorm(hidden, indices.long(), None, float(eps), gathered, normed)
    return [gathered, normed]


def scatter_and_return_cuda(sparse_values: torch.Tensor, indices: torch.Tensor, global_cache: torch.Tensor,
                            current_hidden: torch.Tensor) -> torch.Tensor:
    """Write sparse rows into both the cache and the working hidden tensor; returns
    current_hidden (fused_gather_norm.cu:79-119)."""
    idx = indices.long()
    torch.ops.fdl.kv_scatter(global_cache, current_hidden, sparse_values, sparse_values, idx, 1)
    return current_hidden


def get_fused_ops():
    """Load the native library once and return the ops namespace."""
    global _OPS
    if _OPS is None:
        _lib.ensure_ops()
        _OPS = SimpleNamespace(
            gather_rmsnorm_cuda=gather_rmsnorm_cuda,
            scatter_and_return_cuda=scatter_and_return_cuda,
            fused_select_norm=fused_select_norm,
            fused_gather_input_rmsnorm_pair=fused_gather_input_rmsnorm_pair_raw,
        )
    return _OPS


def fused_gather_input_rmsnorm_pair(
    hidden_states: torch.Tensor,
    token_indices: torch.Tensor,
    input_layernorm: torch.nn.Module,
) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """(selected_hidden, selected_norm) for the rows token_indices of
    hidden_states, or None for non-CUDA input (the caller's torch path)."""
    if not hidden_states.is_cuda:
        return None
    get_fused_ops()
    w = getattr(input_layernorm, "weight", None)
    if w is None:
        return None
    eps = float(getattr(input_layernorm, "variance_epsilon", 1e-6))
    b, _, h = hidden_states.shape
    t = token_indices.shape[1]
    x = hidden_states if hidden_states.stride(-1) == 1 else hidden_states.contiguous()
    gathered, normed = _out(x, b, t, h), _out(x, b, t, h)
    wt = w.detach()
    if wt.dtype != x.dtype:
        # weight * normed.to(dtype) with a weight of another dtype promotes; keep
        # the reference's result dtype by running the product in torch.
        torch.ops.fdl.gather_rmsnorm(x, token_indices.long(), None, eps, gathered, normed)
        return gathered, wt * normed
    torch.ops.fdl.gather_rmsnorm(x, token_indices.long(), wt.contiguous(), eps, gathered, normed)
    return gathered, normed
