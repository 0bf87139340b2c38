"""Drop-in replacements for the reference's utils/ cache and attention modules.

The reference's generation_functions.py imports these submodules by name
(``from utils.static_kv_cache import StaticKVCache, StaticBlockCache`` ...);
see ``fast_v2_b200.dropin.install`` or re-export stubs in the reference tree.
"""
from .attention_backends import (  # noqa: F401
    AttentionBackend,
    get_attention_backend,
    patch_attention_layers,
    patch_attention_layers_compiled,
    unpatch_attention_layers,
)
from .block_sparse_cache import BlockSparseCache  # noqa: F401
from .dynamic_block_kv import DynamicBlockKV  # noqa: F401
from .static_kv_cache import StaticBlockCache, StaticKVCache  # noqa: F401
