"""CPU checks of the native boundary: the C-ABI library loads and exports
every symbol include/fdl_kvcache.h declares; the torch ops register with
Meta kernels (shape inference without a GPU)."""
import re
from pathlib import Path

import torch

from fast_v2_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "fdl_kvcache.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(fdl_\w+)\s*\(", text, re.M)))


def test_header_and_export_list_agree():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.abi()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert _lib.version().startswith("fdl_b200")


def test_host_side_argument_checks_without_gpu():
    # workspace sizing and split choice are pure host logic
    assert _lib.sparse_prefix_workspace_bytes(64, 2080) >= 64 * 2080 * 4
    assert _lib.attn_workspace_bytes(2, 32, 28, 1) == 0
    assert _lib.attn_workspace_bytes(2, 32, 28, 4) >= 4 * 2 * 32 * 28 * 129 * 4
    assert _lib.attn_auto_splits(64, 32, 28, 4, 8224, 0) == 1
    assert _lib.attn_auto_splits(1, 32, 28, 4, 8224, 0) > 1
    # B=16 at a short prefix runs as 128-row CTAs (two 16-query chunks) with
    # no split; at P=8192 it keeps the 256-row form with two KV splits.
    assert _lib.attn_auto_splits(16, 32, 28, 4, 544, 0) == 1
    assert _lib.attn_auto_splits(16, 32, 28, 4, 8224, 0) == 2
    # config 4's geometry (12 query / 2 KV heads): one pass of 96-row CTAs
    # at short prefixes, where splitting 192-row CTAs measured 20-34% slower
    assert _lib.attn_auto_splits(16, 32, 12, 2, 288, 0) == 1
    assert _lib.attn_auto_splits(16, 32, 12, 2, 544, 0) == 1


def test_torch_ops_meta_shapes():
    _lib.ensure_ops()
    m = torch.device("meta")
    q = torch.empty(3, 32, 28, 128, dtype=torch.bfloat16, device=m)
    k = torch.empty(3, 1024, 4, 128, dtype=torch.bfloat16, device=m)
    s = torch.empty(3, dtype=torch.int32, device=m)
    out = torch.ops.fdl.flash_kvcache(q, k, k, s, 0.088, False)
    assert out.shape == q.shape and out.dtype == q.dtype
    for op in ("kv_append", "kv_scatter", "kv_gather_prefix", "kv_gather_rows", "kv_compact", "kv_sparse_prefix",
               "cosine_select", "focus_select", "focus_importance", "rope_qkv_kv",
               "gather_rmsnorm", "block_attn"):
        assert hasattr(torch.ops.fdl, op)
