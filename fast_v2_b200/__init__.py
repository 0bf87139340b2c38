"""fast_v2_b200 -- B200 (sm_100a) KV-cache hot path for Fast-dLLM v2 block diffusion.

Native code lives in two in-tree libraries built by ``fast_v2_b200.build``:
``libfdl_b200.so`` (the C ABI of include/fdl_kvcache.h) and ``libfdl_torch.so``
(torch.ops.fdl registration).  Importing the package does not load them; the
cache/attention classes do on first use and raise ImportError if they are
missing -- there is no CPU or library fallback.
"""
from ._lib import abi, ensure_ops, last_device_error, version  # noqa: F401

__all__ = ["abi", "ensure_ops", "last_device_error", "version"]
