"""Route the reference's module names to this package without editing its files.

    import fast_v2_b200.dropin as d; d.install()

After ``install()``, ``import utils.static_kv_cache`` (and the other four
modules on the hot path) resolve to the B200 implementations, so the
reference's generation_functions.py and eval.py drive them unchanged.  Modules
of the reference that are not on the hot path (utils.batch_bucketing,
utils.dynamo_utils, the model) keep resolving to the reference's own files.
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
