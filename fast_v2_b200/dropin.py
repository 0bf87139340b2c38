"""Route the reference's module names to this package without editing its files.

    import fast_v2_b200.dropin as d; d.install()

After ``install()``, ``import utils.static_kv_cache`` (and the other four
modules on the hot path) resolve to the B200 implementations, so the
reference's generation_functions.py and eval.py drive them unchanged.  Modules
of the reference that are not on the hot path (utils.batch_bucketing,
utils.dynamo_utils, the model) keep resolving to the reference's own files.

The FOCUS token selection lives in module-level helpers of the model file
(modeling.py:214-306); ``patch_modeling(modeling)`` points those names at the
GPU versions in ``fast_v2_b200.focus`` and returns the originals.
"""
from __future__ import annotations

import importlib
import sys

MODULES = {
    "utils.static_kv_cache": "fast_v2_b200.utils.static_kv_cache",
    "utils.dynamic_block_kv": "fast_v2_b200.utils.dynamic_block_kv",
    "utils.block_sparse_cache": "fast_v2_b200.utils.block_sparse_cache",
    "utils.attention_backends": "fast_v2_b200.utils.attention_backends",
    "fused_sparse_extension": "fast_v2_b200.cuda_bench.fused_sparse_extension",
    "cuda_bench.fused_sparse_extension": "fast_v2_b200.cuda_bench.fused_sparse_extension",
}


def install() -> None:
    """Alias the reference's hot-path module names to this package."""
    for ref_name, ours in MODULES.items():
        mod = importlib.import_module(ours)
        sys.modules[ref_name] = mod
        parent, _, child = ref_name.rpartition(".")
        if parent and parent in sys.modules:
            setattr(sys.modules[parent], child, mod)


def uninstall() -> None:
    for ref_name in MODULES:
        sys.modules.pop(ref_name, None)


FOCUS_HELPERS = {"_focus_importance": "focus_importance", "_focus_select": "focus_select"}


def patch_modeling(modeling) -> dict:
    """Swap the FOCUS helpers of a loaded modeling module
    (``_focus_importance``, ``_focus_select``) for the fdl kernels; returns
    the replaced functions so ``unpatch_modeling`` can restore them."""
    from . import focus

    old = {}
    for name, ours in FOCUS_HELPERS.items():
        if hasattr(modeling, name):
            old[name] = getattr(modeling, name)
            setattr(modeling, name, getattr(focus, ours))
    return old


def unpatch_modeling(modeling, old: dict) -> None:
    for name, fn in old.items():
        setattr(modeling, name, fn)
