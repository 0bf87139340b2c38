"""Host-side contracts of the drop-in boundary, checked without a GPU:
reference fallbacks that must stay (None for non-CUDA input), loud failure
instead of a silent CPU path, and C-ABI argument checks that return before
any device work."""
import ctypes

import pytest
import torch

from fast_v2_b200 import _lib
from fast_v2_b200.cuda_bench.fused_sparse_extension import fused_gather_input_rmsnorm_pair
from fast_v2_b200.utils.static_kv_cache import StaticKVCache

FDL_OK, FDL_E_NULL, FDL_E_SHAPE, FDL_E_UNSUPPORTED = 0, 1, 2, 6


class _Norm(torch.nn.Module):
    def __init__(self, h):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(h, dtype=torch.bfloat16), requires_grad=False)
        self.variance_epsilon = 1e-6


def test_fused_pair_returns_none_for_cpu_input_like_the_reference():
    x = torch.randn(2, 16, 64).to(torch.bfloat16)
    idx = torch.tensor([[0, 3], [5, 9]])
    assert fused_gather_input_rmsnorm_pair(x, idx, _Norm(64)) is None


def test_cpu_cache_fails_loudly_instead_of_falling_back():
    cache = StaticKVCache(2, 64, 1, 4, 128, torch.bfloat16, torch.device("cpu"))
    k = torch.zeros(2, 32, 4, 128, dtype=torch.bfloat16)
    with pytest.raises((NotImplementedError, RuntimeError)):
        cache.write_sparse(k, k, 0, torch.zeros(2, 32, dtype=torch.long))


def test_c_abi_argument_checks_return_before_device_work():
    lib = _lib.abi()
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.fdl_gather_rmsnorm.argtypes = [vp, vp, i64, vp, ctypes.c_float, vp, vp, i32, i32, i32, i32, i32, i64, i64,
                                       i64, i64, vp]
    lib.fdl_gather_rmsnorm.restype = i32
    fake = ctypes.c_void_p(0x1000)
    # zero rows: nothing to do, pointers may be NULL
    assert lib.fdl_gather_rmsnorm(None, None, 0, None, 1e-6, None, None, 1, 0, 0, 64, 0, 0, 0, 0, 0, None) == FDL_OK
    # rows to do but no input
    assert lib.fdl_gather_rmsnorm(None, None, 0, None, 1e-6, None, fake, 1, 4, 4, 64, 0, 0, 0, 0, 0,
                                  None) == FDL_E_NULL
    # identity gather asking for more rows than the sequence has
    assert lib.fdl_gather_rmsnorm(fake, None, 0, None, 1e-6, None, fake, 1, 4, 8, 64, 0, 0, 0, 0, 0,
                                  None) == FDL_E_SHAPE
    lib.fdl_swiglu.argtypes = [vp, i64, vp, i64, i64, i32, vp]
    lib.fdl_swiglu.restype = i32
    assert lib.fdl_swiglu(fake, 16, fake, 8, 4, 12, None) == FDL_E_SHAPE  # F not a multiple of 8
    assert lib.fdl_swiglu(None, 16, None, 8, 0, 8, None) == FDL_OK
    lib.fdl_block_attn.argtypes = [vp, vp, vp, vp, i32, vp, vp, i32, vp, i32, vp, i32, i32, i32, i32, i32,
                                   ctypes.c_float] + [i64] * 12 + [i32, vp, i64, vp]
    lib.fdl_block_attn.restype = i32
    args = [fake, fake, fake, fake, 64, None, None, 0, None, 0, fake, 1, 32, 28, 4]
    strides = [0] * 12
    assert lib.fdl_block_attn(*args, 64, 0.125, *strides, 0, None, 0, None) == FDL_E_UNSUPPORTED  # head_dim 64
    assert lib.fdl_block_attn(*args[:12], 32, 27, 4, 128, 0.125, *strides, 0, None, 0, None) == FDL_E_SHAPE
    lib.fdl_kv_compact.argtypes = [vp, i32, i64, i64, i32, vp, i32, vp]
    lib.fdl_kv_compact.restype = i32
    bufs = (ctypes.c_void_p * 2)(0x1000, 0x2000)
    assert lib.fdl_kv_compact(None, 2, 64, 64, 4, None, 0, None) == FDL_OK  # nothing kept: nothing to move
    assert lib.fdl_kv_compact(bufs, 2, 64, 64, 4, None, 3, None) == FDL_E_NULL
    assert lib.fdl_kv_compact(bufs, 2, 64, 64, 4, fake, 5, None) == FDL_E_SHAPE  # more kept rows than slots
    assert lib.fdl_kv_compact(bufs, 2, 64, 32, 4, fake, 3, None) == FDL_E_SHAPE  # rows would overlap
    assert lib.fdl_kv_compact(bufs, 2, 64, 64, 5000, fake, 4097, None) == FDL_E_SHAPE  # list too long
    assert lib.fdl_kv_compact(bufs, 2, 63, 63, 4, fake, 3, None) == 3  # FDL_E_ALIGN: odd row bytes
    # token selection: one block of <= 32 tokens, bf16 (0) or fp32 (2) only
    lib.fdl_focus_select.argtypes = [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, vp, i64, vp, vp]
    lib.fdl_focus_select.restype = i32
    assert lib.fdl_focus_select(None, 32, None, 32, None, 0, 0, 32, 4, 0, None, 32, None, None) == FDL_OK
    assert lib.fdl_focus_select(None, 32, None, 32, None, 0, 2, 32, 4, 0, None, 32, None, None) == FDL_E_NULL
    assert lib.fdl_focus_select(fake, 33, fake, 33, None, 0, 2, 33, 4, 0, fake, 33, fake, None) == FDL_E_SHAPE
    assert lib.fdl_focus_select(fake, 32, fake, 32, None, 0, 2, 32, 0, 0, fake, 32, fake, None) == FDL_E_SHAPE
    assert lib.fdl_focus_select(fake, 32, fake, 32, None, 0, 2, 32, 4, 1, fake, 32, fake, None) == 4  # FDL_E_DTYPE
    lib.fdl_cosine_select.argtypes = [vp, vp, vp, i32, i32, i32, i32] + [i64] * 6 + [i32, vp, i64, vp, vp]
    lib.fdl_cosine_select.restype = i32
    st = [32 * 64, 64, 32 * 64, 64, 0, 0]
    assert lib.fdl_cosine_select(fake, fake, None, 2, 32, 60, 0, *st, 8, fake, 8, None, None) == FDL_E_SHAPE
    assert lib.fdl_cosine_select(fake, fake, None, 2, 32, 64, 0, *st, 33, fake, 33, None, None) == FDL_E_SHAPE
    assert lib.fdl_cosine_select(None, fake, None, 2, 32, 64, 0, *st, 8, fake, 8, None, None) == FDL_E_NULL
    assert lib.fdl_cosine_select(fake, fake, None, 2, 32, 64, 0, 32 * 64, 60, 32 * 64, 64, 0, 0, 8, fake, 8, None,
                                 None) == 3  # FDL_E_ALIGN: token stride of 120 bytes
    lib.fdl_focus_importance.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32] + [i64] * 7 + [ctypes.c_float, vp,
                                                                                             i64, vp]
    lib.fdl_focus_importance.restype = i32
    ist = [0] * 7
    assert lib.fdl_focus_importance(fake, fake, fake, 1, 32, 28, 3, 128, 0, *ist, 0.1, fake, 32, None) == FDL_E_SHAPE
    assert lib.fdl_focus_importance(fake, fake, fake, 1, 32, 28, 4, 256, 0, *ist, 0.1, fake, 32, None) == FDL_E_SHAPE
    assert lib.fdl_focus_importance(fake, fake, None, 1, 32, 28, 4, 128, 0, *ist, 0.1, fake, 32, None) == FDL_E_NULL


def test_compaction_index_checks_run_on_the_host():
    """compact_batch validates active_indices before any device work: the
    in-place order needs i <= active_indices[i] < batch for every i."""
    from fast_v2_b200.utils.compaction import active_rows, regrow

    act = active_rows(torch.tensor([1, 2, 4], dtype=torch.int32), 5, "cpu")
    assert act.dtype == torch.int64 and act.tolist() == [1, 2, 4]
    assert active_rows([3, 1], 4, "cpu").tolist() == [3, 1]  # out of order but still in place-safe
    assert active_rows(torch.empty(0, dtype=torch.long), 4, "cpu").numel() == 0
    for bad, batch in (([1, 0], 4), ([0, 4], 4), ([0, 1, 2], 2)):
        with pytest.raises(ValueError):
            active_rows(torch.tensor(bad), batch, "cpu")
    with pytest.raises(ValueError):
        active_rows(torch.tensor([True, False, True]), 3, "cpu")
    # regrow: a prefix view grows back over its own storage, zeroed
    full = torch.arange(24, dtype=torch.float32).reshape(6, 4)
    grown = regrow(full[:2], 6)
    assert grown.data_ptr() == full.data_ptr() and grown.shape == (6, 4) and int(full.abs().sum()) == 0
    lone = torch.ones(2, 4)
    assert regrow(lone, 6).shape == (6, 4) and int(regrow(lone, 6).sum()) == 0
    bsc = torch.ones(3, 5, 2)
    g2 = regrow(bsc[:, :2], 5, dim=1)
    assert g2.shape == (3, 5, 2) and g2.data_ptr() == bsc.data_ptr() and int(bsc.sum()) == 0


def test_module_aliasing_and_modeling_patch():
    """install() makes the reference's hot-path module names resolve to this
    package; patch_modeling() swaps the FOCUS helpers by name and restores them."""
    import importlib
    import sys
    import types

    from fast_v2_b200 import dropin, focus
    from fast_v2_b200.utils import static_kv_cache as ours

    dropin.install()
    try:
        mod = importlib.import_module("utils.static_kv_cache")
        assert mod is ours and mod.StaticKVCache is ours.StaticKVCache
        assert sys.modules["fused_sparse_extension"].fused_gather_input_rmsnorm_pair is not None
    finally:
        dropin.uninstall()
    assert "utils.static_kv_cache" not in sys.modules
    modeling = types.ModuleType("fake_modeling")
    modeling._focus_select = orig_sel = lambda *a, **k: None
    modeling._focus_importance = orig_imp = lambda *a, **k: None
    old = dropin.patch_modeling(modeling)
    assert modeling._focus_select is focus.focus_select and modeling._focus_importance is focus.focus_importance
    dropin.unpatch_modeling(modeling, old)
    assert modeling._focus_select is orig_sel and modeling._focus_importance is orig_imp
