"""The allocation-free entry point fdl_kv_sparse_prefix_noalloc.

Some callers of this library cannot allocate device memory themselves: code
that runs inside another framework's memory pool, services that forbid
cudaMalloc once they are up, or thin bindings that only pass the tensors they
already own.  For them the key-norm prefix selection keeps its score scratch
in a fixed array inside the library instead of a caller-supplied workspace.

This file is collected last on purpose.  It calls the entry point through the
C ABI (ctypes), twice in a row with different inputs (the shared scratch keeps
the previous call's contents), and checks both results against the existing
entry point fdl_kv_sparse_prefix (through torch.ops.fdl) -- selection and
gather are bit-exact, so the comparison is exact.  It also checks that a
request larger than the array is refused with FDL_E_WORKSPACE.
"""
import ctypes

import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
FDL_E_WORKSPACE = 5
NOALLOC_MAX = 1 << 20


def _noalloc_fn():
    lib = _lib.abi()
    f = lib.fdl_kv_sparse_prefix_noalloc
    i32, i64, vp = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p
    f.argtypes = [vp, vp, vp, i32, i32, i32, i32, i64, i64, i64, i32, i32, i32, vp, vp, vp, vp, i64, i64, i64, vp]
    f.restype = i32
    return f


def _inputs(seed, B, cap, lens):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, cap, 4, 128, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, cap, 4, 128, generator=g).to(torch.bfloat16).to(DEV)
    k[0, 7] = k[0, 3]  # a tie: the lower index must win
    return k, v, torch.tensor(lens, dtype=torch.int32, device=DEV)


def _run_noalloc(f, k, v, lens, max_keep):
    B, cap, H, D = k.shape
    sel = torch.full((B, max_keep), -7, dtype=torch.int32, device=DEV)
    out_len = torch.full((B,), -7, dtype=torch.int32, device=DEV)
    ko = torch.zeros(B, max_keep, H, D, dtype=torch.bfloat16, device=DEV)
    vo = torch.zeros_like(ko)
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(k.data_ptr(), v.data_ptr(), lens.data_ptr(), B, cap, H, D, *k.stride()[:3], 1, 4, max_keep,
           sel.data_ptr(), out_len.data_ptr(), ko.data_ptr(), vo.data_ptr(), *ko.stride()[:3], stream)
    assert rc == 0, f"fdl_kv_sparse_prefix_noalloc returned {rc}"
    return sel, out_len, ko, vo


def _run_existing(k, v, lens, max_keep):
    B, cap, H, D = k.shape
    sel = torch.empty(B, max_keep, dtype=torch.int32, device=DEV)
    out_len = torch.empty(B, dtype=torch.int32, device=DEV)
    ko = torch.zeros(B, max_keep, H, D, dtype=torch.bfloat16, device=DEV)
    vo = torch.zeros_like(ko)
    ws = torch.empty(_lib.sparse_prefix_workspace_bytes(B, cap), dtype=torch.uint8, device=DEV)
    torch.ops.fdl.kv_sparse_prefix(k, v, lens, 1, 4, sel, out_len, ko, vo, ws)
    return sel, out_len, ko, vo


def test_noalloc_matches_existing_entry_point_on_two_calls():
    _lib.ensure_ops()
    f = _noalloc_fn()
    cases = [(11, 4, 2048, [2048, 1500, 0, 257]),   # first call
             (12, 3, 1000, [999, 1, 640])]           # second call, different shape, stale scratch behind it
    for seed, B, cap, lens in cases:
        k, v, L = _inputs(seed, B, cap, lens)
        max_keep = max(1, -(-max(lens) // 4))
        got = _run_noalloc(f, k, v, L, max_keep)
        ref = _run_existing(k, v, L, max_keep)
        torch.cuda.synchronize()
        assert torch.equal(got[1], ref[1]), "kept counts differ"
        assert torch.equal(got[0], ref[0]), "selected indices differ"
        for b in range(B):
            n = int(ref[1][b])
            assert torch.equal(got[2][b, :n], ref[2][b, :n]) and torch.equal(got[3][b, :n], ref[3][b, :n])
        s0 = set(got[0][0, : int(ref[1][0])].cpu().tolist())
        assert not (7 in s0 and 3 not in s0)  # equal scores: the lower index wins
    code, info = _lib.last_device_error()
    assert code == 0, (code, info)


def test_noalloc_rejects_requests_beyond_its_scratch():
    f = _noalloc_fn()
    B, cap = 64, NOALLOC_MAX // 64 + 1
    dummy = torch.zeros(16, dtype=torch.uint8, device=DEV)
    p = dummy.data_ptr()
    rc = f(p, p, p, B, cap, 4, 128, cap * 512, 512, 128, 1, 4, 8, p, p, p, p, 8 * 512, 512, 128,
           torch.cuda.current_stream().cuda_stream)
    assert rc == FDL_E_WORKSPACE
    torch.cuda.synchronize()
    assert np.all(dummy.cpu().numpy() == 0)  # nothing was launched
