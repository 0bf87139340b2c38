"""Edge cases of the hot path on the GPU: empty work, the cache's last rows,
sequences with nothing to attend to, and size limits.  Each case is checked
against the oracle (bit-exact for copies) or against its defined result."""
import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib
from oracle import kvcache_oracle as O
from tests._util import assert_close, bits_of

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rbf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _clean_status():
    code, _ = _lib.last_device_error()
    return code == 0


def test_append_of_zero_tokens_is_a_no_op():
    k = rbf16((2, 64, 4, 128), 1).to(DEV)
    v = rbf16((2, 64, 4, 128), 2).to(DEV)
    k0, v0 = k.clone(), v.clone()
    src = torch.empty(2, 0, 4, 128, dtype=torch.bfloat16, device=DEV)
    torch.ops.fdl.kv_append([k], [v], [src], [src], torch.tensor([3, 64], dtype=torch.int32, device=DEV))
    assert torch.equal(k, k0) and torch.equal(v, v0) and _clean_status()


def test_append_filling_the_last_rows_of_the_cache():
    B, S, H, D, n = 3, 96, 4, 128, 32
    kc, vc = rbf16((B, S, H, D), 3), rbf16((B, S, H, D), 4)
    ks, vs = rbf16((B, n, H, D), 5), rbf16((B, n, H, D), 6)
    start = np.array([S - n, 0, S - n], np.int32)
    gk, gv = kc.to(DEV), vc.to(DEV)
    torch.ops.fdl.kv_append([gk], [gv], [ks.to(DEV)], [vs.to(DEV)], torch.from_numpy(start).to(DEV))
    ek, ev = bits_of(kc).copy(), bits_of(vc).copy()
    O.kv_append(ek, ev, bits_of(ks), bits_of(vs), start)
    assert np.array_equal(bits_of(gk), ek) and np.array_equal(bits_of(gv), ev) and _clean_status()


def test_scatter_of_zero_positions_is_a_no_op():
    dst = rbf16((2, 4, 32, 128), 7).to(DEV)
    d0 = dst.clone()
    src = torch.empty(2, 4, 0, 128, dtype=torch.bfloat16, device=DEV)
    pos = torch.empty(2, 0, dtype=torch.int64, device=DEV)
    torch.ops.fdl.kv_scatter(dst, None, src, None, pos, 2)
    assert torch.equal(dst, d0) and _clean_status()


def test_gather_prefix_of_all_empty_sequences():
    B, S, H, D = 3, 64, 4, 128
    kc, vc = rbf16((B, S, H, D), 8).to(DEV), rbf16((B, S, H, D), 9).to(DEV)
    lens = torch.zeros(B, dtype=torch.int32, device=DEV)
    cu = torch.zeros(B + 1, dtype=torch.int32, device=DEV)
    ok = torch.empty(0, H * 7, D, dtype=torch.bfloat16, device=DEV)
    ov = torch.empty_like(ok)
    torch.ops.fdl.kv_gather_prefix(kc, vc, lens, None, None, 7, ok, ov, cu, 1, 1)
    assert _clean_status()


def test_norms_and_elementwise_ops_on_zero_rows():
    H = 3584
    x = torch.empty(0, H, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(H, dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(x)
    torch.ops.fdl.add_rmsnorm(x, x.clone(), w, 1e-6, None, out)
    torch.ops.fdl.gather_rmsnorm(x.view(1, 0, H), None, w, 1e-6, None, out.view(1, 0, H))
    torch.ops.fdl.swiglu(torch.empty(0, 2 * 64, dtype=torch.bfloat16, device=DEV),
                         torch.empty(0, 64, dtype=torch.bfloat16, device=DEV))
    assert _clean_status()


def test_gather_rmsnorm_first_and_last_rows_and_no_weight():
    B, S, H = 2, 50, 3584
    x = rbf16((B, S, H), 10)
    idx = np.array([[0, S - 1, 7], [S - 1, 0, 0]], np.int64)
    gath = torch.empty(B, 3, H, dtype=torch.bfloat16, device=DEV)
    normed = torch.empty_like(gath)
    torch.ops.fdl.gather_rmsnorm(x.to(DEV), torch.from_numpy(idx).to(DEV), None, 1e-6, gath, normed)
    eg, en = O.gather_rmsnorm_bf16(bits_of(x), idx, None, 1e-6)
    assert np.array_equal(bits_of(gath), eg)
    assert_close("no-weight norm", normed.float().cpu().numpy(), O.bf16_to_f32(en), 2e-2, 1e-2)


def test_attention_with_every_sequence_empty_gives_zeros():
    B, Sq, Hq, Hkv, cap = 3, 32, 28, 4, 256
    q = rbf16((B, Sq, Hq, 128), 11, 128 ** -0.5).to(DEV)
    k = rbf16((B, cap, Hkv, 128), 12).to(DEV)
    v = rbf16((B, cap, Hkv, 128), 13).to(DEV)
    seq = torch.zeros(B, dtype=torch.int32, device=DEV)
    out = torch.full_like(q, 7.0)
    torch.ops.fdl.block_attn(q, k, v, seq, None, None, None, 0, 128 ** -0.5, out, None, 1)
    assert float(out.float().abs().max()) == 0.0 and _clean_status()


@pytest.mark.parametrize("lens", [[1, 1], [128, 129], [255, 1]])
def test_attention_at_tile_boundaries(lens):
    """Lengths 1, one tile exactly, one past a tile: the edge-tile path."""
    B, Sq, Hq, Hkv, cap = len(lens), 32, 28, 4, 256
    q = rbf16((B, Sq, Hq, 128), 14, 128 ** -0.5)
    k, v = rbf16((B, cap, Hkv, 128), 15), rbf16((B, cap, Hkv, 128), 16)
    out = torch.empty(B, Sq, Hq, 128, dtype=torch.bfloat16, device=DEV)
    torch.ops.fdl.block_attn(q.to(DEV), k.to(DEV), v.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV),
                             None, None, None, 0, 128 ** -0.5, out, None, 1)
    ref = O.block_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), lens)
    assert_close("attn edge", out.float().cpu().numpy(), ref, 2e-2, 1e-2)


def test_attention_length_beyond_capacity_is_clamped_and_reported():
    B, Sq, Hq, Hkv, cap = 1, 8, 28, 4, 128
    q = rbf16((B, Sq, Hq, 128), 17, 128 ** -0.5)
    k, v = rbf16((B, cap, Hkv, 128), 18), rbf16((B, cap, Hkv, 128), 19)
    out = torch.empty(B, Sq, Hq, 128, dtype=torch.bfloat16, device=DEV)
    torch.ops.fdl.block_attn(q.to(DEV), k.to(DEV), v.to(DEV), torch.tensor([cap + 50], dtype=torch.int32, device=DEV),
                             None, None, None, 0, 128 ** -0.5, out, None, 1)
    code, info = _lib.last_device_error()
    assert code == 2 and info == cap + 50  # FDL_DEV_LENGTH, the offending length
    ref = O.block_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), [cap])
    assert_close("clamped", out.float().cpu().numpy(), ref, 2e-2, 1e-2)
