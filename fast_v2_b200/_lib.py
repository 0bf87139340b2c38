"""Loading of the in-tree native libraries.

``abi()`` returns a :class:`ctypes.CDLL` for ``libfdl_b200.so`` (the C ABI of
``include/fdl_kvcache.h``); ``ensure_ops()`` registers the ``torch.ops.fdl``
operators from ``libfdl_torch.so``.  There is no fallback: if a library is
missing or fails to load, an ``ImportError`` names the file and the command
that builds it.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_ABI = PKG / "libfdl_b200.so"
LIB_TORCH = PKG / "libfdl_torch.so"

# Every symbol declared in include/fdl_kvcache.h.
EXPORTS = (
    "fdl_kv_append",
    "fdl_kv_scatter",
    "fdl_kv_gather_prefix",
    "fdl_kv_gather_rows",
    "fdl_kv_compact",
    "fdl_sparse_prefix_workspace_bytes",
    "fdl_kv_sparse_prefix",
    "fdl_kv_sparse_prefix_noalloc",
    "fdl_gather_rmsnorm",
    "fdl_block_attn_workspace_bytes",
    "fdl_block_attn_auto_splits",
    "fdl_block_attn",
    "fdl_rope_qkv",
    "fdl_rope_qkv_kv",
    "fdl_swiglu",
    "fdl_add_rmsnorm",
    "fdl_cosine_select",
    "fdl_focus_select",
    "fdl_focus_importance",
    "fdl_softmax_argmax",
    "fdl_last_device_error",
    "fdl_version",
)

_lock = threading.Lock()
# Host-side tally of fdl kernel launches issued by the Python drivers (a CUDA
# graph replay adds the count recorded at its capture); bench.py reports it.
launches = 0


def count_launches(n: int = 1) -> None:
    global launches
    launches += n

_abi: ctypes.CDLL | None = None
_ops_loaded = False


def _missing(path: Path) -> ImportError:
    return ImportError(
        f"fast_v2_b200: native library {path.name} not found at {path}; "
        f"build it with `python -m fast_v2_b200.build` (nvcc, sm_100a)."
    )


def abi() -> ctypes.CDLL:
    global _abi
    with _lock:
        if _abi is None:
            if not LIB_ABI.exists():
                raise _missing(LIB_ABI)
            lib = ctypes.CDLL(str(LIB_ABI), mode=ctypes.RTLD_GLOBAL)
            i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
            lib.fdl_version.restype = ctypes.c_char_p
            lib.fdl_sparse_prefix_workspace_bytes.restype = i64
            lib.fdl_sparse_prefix_workspace_bytes.argtypes = [i32, i32]
            lib.fdl_block_attn_workspace_bytes.restype = i64
            lib.fdl_block_attn_workspace_bytes.argtypes = [i32, i32, i32, i32, i32]
            lib.fdl_block_attn_auto_splits.restype = i32
            lib.fdl_block_attn_auto_splits.argtypes = [i32] * 6
            lib.fdl_last_device_error.restype = i32
            lib.fdl_last_device_error.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(i64)]
            del vp
            _abi = lib
        return _abi


def ensure_ops() -> None:
    """Register torch.ops.fdl.* (idempotent)."""
    global _ops_loaded
    if _ops_loaded:
        return
    abi()  # libfdl_torch.so resolves its C-ABI symbols from the loaded library
    with _lock:
        if _ops_loaded:
            return
        if not LIB_TORCH.exists():
            raise _missing(LIB_TORCH)
        import torch

        torch.ops.load_library(str(LIB_TORCH))
        _ops_loaded = True


def version() -> str:
    return abi().fdl_version().decode()


def last_device_error() -> tuple[int, int]:
    """(code, info) of the first device-side error since the last call; clears it.

    Synchronises the current device.  Codes: 0 ok, 1 index out of range,
    2 length out of range, 3 pipeline wait timed out.
    """
    code = ctypes.c_int32(0)
    info = ctypes.c_int64(0)
    rc = abi().fdl_last_device_error(ctypes.byref(code), ctypes.byref(info))
    if rc != 0:
        raise RuntimeError(f"fdl_last_device_error failed with CUDA error {-rc}")
    return int(code.value), int(info.value)


class DeviceError(RuntimeError):
    """A kernel of the library recorded a device-side error (an index or
    length outside its buffer, or a pipeline wait that gave up)."""

    def __init__(self, where: str, code: int, info: int):
        self.code, self.info = code, info
        super().__init__(f"{where}: device status {DEVICE_CODES.get(code, code)} (info {info})")


DEVICE_CODES = {1: "FDL_DEV_INDEX: a position or index outside its buffer (the row was skipped)",
                2: "FDL_DEV_LENGTH: a per-sequence length outside [0, capacity] (clamped)",
                3: "FDL_DEV_TIMEOUT: a pipeline wait gave up; the attention output is incomplete"}


def check_device(where: str) -> None:
    """Raise DeviceError if any kernel recorded a device-side error since the
    last check (synchronises the current device and clears the status)."""
    code, info = last_device_error()
    if code != 0:
        raise DeviceError(where, code, info)


def sparse_prefix_workspace_bytes(batch: int, cap: int) -> int:
    return int(abi().fdl_sparse_prefix_workspace_bytes(batch, cap))


def attn_workspace_bytes(batch: int, sq: int, hq: int, num_splits: int) -> int:
    return int(abi().fdl_block_attn_workspace_bytes(batch, sq, hq, 128, num_splits))


def attn_auto_splits(batch: int, sq: int, hq: int, hkv: int, cap: int, n_blk: int) -> int:
    return int(abi().fdl_block_attn_auto_splits(batch, sq, hq, hkv, cap, n_blk))
