"""Parity at the shapes bench.py measures (3 and the
attention launches of config 5).

Every case launches the full grid -- all sequences, every wave, the split-KV
combine where the library picks it -- and compares a sample of sequences
spread over the batch against the CPU oracle (float64 attention; bit-exact
copies).  Properties that need no oracle (nothing outside an append window
changes; each packed sequence equals its GQA-expanded cache rows) are checked
on the whole output.  Tolerances: max-abs 2e-2 + rel 1e-2 for attention in
bf16; bit-exact for append and gather."""
import math

import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib
from oracle import kvcache_oracle as O
from tests._util import assert_close, bits_of

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
DEV = "cuda"
HQ, HKV, D = 28, 4, 128


@pytest.fixture(autouse=True)
def _ops():
    _lib.ensure_ops()
    _lib.last_device_error()
    yield
    code, info = _lib.last_device_error()
    assert code == 0, f"device error {code} (info {info}) left by the test"


def _sample(B):
    """Up to 4 sequences spread over the batch (first, last and two inside)."""
    return sorted({0, B // 3, (2 * B) // 3, B - 1})


def _attn(q, k, v, seq, kb=None, vb=None, q_pos=None, mask_block=0):
    B, Sq, Hq, _ = q.shape
    ns = _lib.attn_auto_splits(B, Sq, Hq, k.shape[2], k.shape[1], kb.shape[1] if kb is not None else 0)
    wsb = _lib.attn_workspace_bytes(B, Sq, Hq, ns)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV) if wsb > 0 else None
    out = torch.empty_like(q)
    torch.ops.fdl.block_attn(q, k, v, seq, kb, vb, q_pos, mask_block, D ** -0.5, out, ws, ns)
    return out, ns


# ------------------------------------------------------------ config 3
@pytest.mark.parametrize("Sq", [32, 8])
@pytest.mark.parametrize("P", [512, 2048, 8192])
@pytest.mark.parametrize("B", [1, 16, 64])
def test_block_attn_config3_grid(B, P, Sq):
    """Q [B, Sq, 28, 128] ~ N(0,1)/sqrt(128) over K/V [B, P+32, 4, 128] ~ N(0,1),
    every key valid (cache_seqlens = P + 32), the library's own split choice."""
    cap = P + 32
    g = torch.Generator(device=DEV).manual_seed(3000 + 7 * B + P + Sq)
    q = (torch.randn(B, Sq, HQ, D, generator=g, device=DEV) / math.sqrt(D)).to(torch.bfloat16)
    k = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    seq = torch.full((B,), cap, dtype=torch.int32, device=DEV)
    out, ns = _attn(q, k, v, seq)
    assert torch.isfinite(out.float()).all()
    for b in _sample(B):
        ref = O.block_attention(q[b:b + 1].float().cpu().numpy(), k[b:b + 1].float().cpu().numpy(),
                                v[b:b + 1].float().cpu().numpy(), [cap])
        assert_close(f"B={B} P={P} Sq={Sq} splits={ns} b={b}", out[b:b + 1].float().cpu().numpy(), ref, ATOL, RTOL)


@pytest.mark.parametrize("splits", [0, 4])
@pytest.mark.parametrize("mask", [0, 32])
def test_block_attn_config4_geometry(mask, splits):
    """Config 4's attention (Qwen2.5-1.5B: 12 query heads over 2 KV heads, 16
    sequences, 32 queries over cache[:len + 32] with ragged lengths), without
    the static schedule's mask (mask 0) and with the block-causal one (queries
    at positions len..len+31).  The library's own choice (splits 0) runs
    128-row CTAs (6 heads x 16 queries = 96 rows: one row tile with a whole
    padding warp) without a split; with four splits forced it runs 256-row
    CTAs (6 x 32 = 192 rows, the second row tile half padding) and the
    combine pass."""
    B, Sq, Hq, Hkv = 16, 32, 12, 2
    g = torch.Generator(device=DEV).manual_seed(3400 + mask)
    lens = torch.randint(200, 800, (B,), generator=g, device=DEV)
    cap = int(lens.max()) + 32 + 64
    q = (torch.randn(B, Sq, Hq, D, generator=g, device=DEV) / math.sqrt(D)).to(torch.bfloat16)
    k = torch.randn(B, cap, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, cap, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    seq = (lens + 32).to(torch.int32)
    q_pos = (lens[:, None] + torch.arange(Sq, device=DEV)[None, :]).to(torch.int32).contiguous()
    ns = splits or _lib.attn_auto_splits(B, Sq, Hq, Hkv, cap, 0)
    wsb = _lib.attn_workspace_bytes(B, Sq, Hq, ns)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV) if wsb > 0 else None
    out = torch.empty_like(q)
    torch.ops.fdl.block_attn(q, k, v, seq, None, None, q_pos if mask else None, mask, D ** -0.5, out, ws, ns)
    for b in _sample(B):
        n = int(seq[b])
        qp = q_pos[b].cpu().numpy() if mask else None
        ref = O.block_attention(q[b:b + 1].float().cpu().numpy(), k[b:b + 1, :n].float().cpu().numpy(),
                                v[b:b + 1, :n].float().cpu().numpy(), [n],
                                **({"q_pos": qp[None, :], "mask_block": mask} if mask else {}))
        assert_close(f"config4 mask={mask} splits={ns} b={b}", out[b:b + 1].float().cpu().numpy(), ref, ATOL, RTOL)


@pytest.mark.parametrize("B,P", [(16, 8192), (64, 2048)])
def test_block_attn_config3_ragged_lengths(B, P):
    """Same grid points with per-sequence lengths drawn from [1, P+32] (partial
    last tiles, CTAs of one wave finishing at different times)."""
    cap = P + 32
    g = torch.Generator(device=DEV).manual_seed(3100 + B)
    q = (torch.randn(B, 32, HQ, D, generator=g, device=DEV) / math.sqrt(D)).to(torch.bfloat16)
    k = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    lens = torch.randint(1, cap + 1, (B,), generator=torch.Generator().manual_seed(B), dtype=torch.int32)
    out, ns = _attn(q, k, v, lens.to(DEV))
    for b in _sample(B):
        L = int(lens[b])
        ref = O.block_attention(q[b:b + 1].float().cpu().numpy(), k[b:b + 1, :L].float().cpu().numpy(),
                                v[b:b + 1, :L].float().cpu().numpy(), [L])
        assert_close(f"ragged B={B} b={b} L={L} splits={ns}", out[b:b + 1].float().cpu().numpy(), ref, ATOL, RTOL)


# ------------------------------------------------- config 5 attention
@pytest.mark.parametrize("fed", [None, 13])
def test_block_attn_e2e_7b_shape(fed):
    """The attention launches of the default e2e bench: 64 sequences over a
    token-sparse prefix of ~25% of 1024-2048 committed tokens, plus the 32-key
    dKV block buffer (BHSD, a second key source), block-causal mask 32.  A
    full step feeds all 32 block positions; a cached step feeds `fed` of them
    at their own positions."""
    B, nb = 64, 32
    gen = torch.Generator().manual_seed(5000 + (fed or 0))
    lens = torch.randint(256, 513, (B,), generator=gen, dtype=torch.int32)
    cap = 576
    g = torch.Generator(device=DEV).manual_seed(5001)
    k = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    kb = torch.randn(B, HKV, nb, D, generator=g, device=DEV).to(torch.bfloat16)  # BHSD block buffer
    vb = torch.randn(B, HKV, nb, D, generator=g, device=DEV).to(torch.bfloat16)
    # The decoder passes absolute positions: committed length (a multiple of
    # the block) + offset in the block.
    committed = 1024 + 32 * torch.randint(0, 32, (B,), generator=gen)
    if fed is None:
        offs = torch.arange(nb).expand(B, -1)
    else:
        offs = torch.stack([torch.sort(torch.randperm(nb, generator=gen)[:fed]).values for _ in range(B)])
    Sq = offs.shape[1]
    qpos = (committed[:, None] + offs).to(torch.int32)
    q = (torch.randn(B, Sq, HQ, D, generator=g, device=DEV) / math.sqrt(D)).to(torch.bfloat16)
    out, ns = _attn(q, k, v, lens.to(DEV), kb.transpose(1, 2), vb.transpose(1, 2), qpos.to(DEV), 32)
    for b in _sample(B):
        L = int(lens[b])
        ref = O.block_attention(q[b:b + 1].float().cpu().numpy(), k[b:b + 1, :L].float().cpu().numpy(),
                                v[b:b + 1, :L].float().cpu().numpy(), [L],
                                k_blk=kb[b:b + 1].transpose(1, 2).float().cpu().numpy(),
                                v_blk=vb[b:b + 1].transpose(1, 2).float().cpu().numpy(), mask_block=32,
                                q_pos=qpos[b:b + 1].numpy())
        assert_close(f"e2e fed={fed} b={b} L={L}", out[b:b + 1].float().cpu().numpy(), ref, ATOL, RTOL)


# ------------------------------------------------------------ config 2
def test_kv_path_config2_shape():
    """28 layers, B=16, cache [16, 4096, 4, 128] per layer and K/V, lengths
    U[256, 2048] (the bench's seed), one 32-token block appended per sequence
    at its own length, then the packed varlen gather of prefix + block with
    GQA-7 expansion (cu_seqlens int32)."""
    L, B, S, n, rep = 28, 16, 4096, 32, 7
    lens = torch.randint(256, 2049, (B,), generator=torch.Generator().manual_seed(2000), dtype=torch.int32)
    g = torch.Generator(device=DEV).manual_seed(2001)
    kc = [torch.randn(B, S, HKV, D, generator=g, device=DEV).to(torch.bfloat16) for _ in range(L)]
    vc = [torch.randn(B, S, HKV, D, generator=g, device=DEV).to(torch.bfloat16) for _ in range(L)]
    kn = [torch.randn(B, n, HKV, D, generator=g, device=DEV).to(torch.bfloat16) for _ in range(L)]
    vn = [torch.randn(B, n, HKV, D, generator=g, device=DEV).to(torch.bfloat16) for _ in range(L)]
    sample_l = [0, 13, L - 1]
    sample_b = _sample(B)
    before_k = [t.clone() for t in kc]
    before_v = [t.clone() for t in vc]
    torch.ops.fdl.kv_append(kc, vc, kn, vn, lens.to(DEV))
    assert _lib.last_device_error()[0] == 0

    # (1) oracle, bit-exact, on sampled layers x sequences (whole rows).
    for l in sample_l:
        ek, ev = bits_of(before_k[l][sample_b]).copy(), bits_of(before_v[l][sample_b]).copy()
        O.kv_append(ek, ev, bits_of(kn[l][sample_b]), bits_of(vn[l][sample_b]), lens.numpy()[sample_b])
        assert np.array_equal(bits_of(kc[l][sample_b]), ek), f"append K layer {l}"
        assert np.array_equal(bits_of(vc[l][sample_b]), ev), f"append V layer {l}"
    # (2) every layer and sequence: the window holds the new block and nothing
    # outside it changed.
    for l in range(L):
        for b in range(B):
            s0 = int(lens[b])
            before_k[l][b, s0:s0 + n] = kn[l][b]
            before_v[l][b, s0:s0 + n] = vn[l][b]
        assert torch.equal(kc[l], before_k[l]) and torch.equal(vc[l], before_v[l]), f"append layer {l}"
    del before_k, before_v

    after = lens + n
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(after, 0)
    total = int(cu[-1])
    ok = torch.empty(total, HKV * rep, D, dtype=torch.bfloat16, device=DEV)
    ov = torch.empty_like(ok)
    for l in range(L):
        torch.ops.fdl.kv_gather_prefix(kc[l], vc[l], after.to(DEV), None, None, rep, ok, ov, cu.to(DEV), 1, 1)
        if l in sample_l:
            ck = bits_of(kc[l])
            ek, ecu = O.gather_prefix_packed(ck, after.numpy(), rep)
            assert np.array_equal(ecu, cu.numpy())
            assert np.array_equal(bits_of(ok), ek), f"gather K layer {l}"
            ev, _ = O.gather_prefix_packed(bits_of(vc[l]), after.numpy(), rep)
            assert np.array_equal(bits_of(ov), ev), f"gather V layer {l}"
        else:
            for b in range(B):
                a, e = int(cu[b]), int(cu[b + 1])
                assert torch.equal(ok[a:e], kc[l][b, :e - a].repeat_interleave(rep, dim=1)), (l, b)
                assert torch.equal(ov[a:e], vc[l][b, :e - a].repeat_interleave(rep, dim=1)), (l, b)
    assert _lib.last_device_error()[0] == 0


def test_packed_gather_rejects_an_inconsistent_cu_seqlens():
    """A packed range too short for len + n_blk rows, or one past the output,
    is skipped whole and reported -- nothing is written out of range."""
    B, S = 3, 256
    g = torch.Generator(device=DEV).manual_seed(9)
    kc = torch.randn(B, S, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(B, S, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    lens = torch.tensor([100, 50, 80], dtype=torch.int32, device=DEV)
    # Sequence 1's range [100, 140) holds 40 rows but needs 50.
    cu = torch.tensor([0, 100, 140, 220], dtype=torch.int32, device=DEV)
    guard = 64
    ok = torch.zeros(220 + guard, HKV, D, dtype=torch.bfloat16, device=DEV)
    ov = torch.zeros_like(ok)
    torch.ops.fdl.kv_gather_prefix(kc, vc, lens, None, None, 1, ok[:220], ov[:220], cu, 1, 1)
    code, info = _lib.last_device_error()
    assert code == 1 and info == 1
    assert torch.equal(ok[:100], kc[0, :100])
    assert float(ok[100:140].float().abs().max()) == 0.0  # skipped whole
    assert torch.equal(ok[140:220], kc[2, :80])
    assert float(ok[220:].float().abs().max()) == 0.0
    # A range that reaches past the output's rows.
    cu2 = torch.tensor([0, 100, 150, 240], dtype=torch.int32, device=DEV)
    ok.zero_()
    torch.ops.fdl.kv_gather_prefix(kc, vc, lens, None, None, 1, ok[:220], ov[:220], cu2, 1, 1)
    code, info = _lib.last_device_error()
    assert code == 1 and info == 2
    assert float(ok[150:].float().abs().max()) == 0.0


@pytest.mark.parametrize("Sq,n_blk,splits", [(32, 32, 0), (13, 32, 0), (8, 0, 0), (32, 0, 2)])
def test_block_attn_persistent_items_with_empty_and_tiny_sequences(Sq, n_blk, splits):
    """More work items than SMs with a few key tiles each puts the kernel on
    its persistent path (one CTA per SM walking several items).  Sequences of
    length 0 (items with no prefix tiles, or none at all without a block),
    length 1 and lengths straddling tile boundaries are mixed so consecutive
    items of one CTA differ in tile count; with splits=2 items of one sequence
    land on different CTAs and go through the combine."""
    B, cap = 96, 512
    g = torch.Generator(device=DEV).manual_seed(6000 + Sq + n_blk + splits)
    lens = torch.tensor([[0, 1, 127, 128, 129, 300, 511, 512][i % 8] for i in range(B)], dtype=torch.int32)
    q = (torch.randn(B, Sq, HQ, D, generator=g, device=DEV) / math.sqrt(D)).to(torch.bfloat16)
    k = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, cap, HKV, D, generator=g, device=DEV).to(torch.bfloat16)
    kb = vb = None
    if n_blk:
        kb = torch.randn(B, HKV, n_blk, D, generator=g, device=DEV).to(torch.bfloat16).transpose(1, 2)
        vb = torch.randn(B, HKV, n_blk, D, generator=g, device=DEV).to(torch.bfloat16).transpose(1, 2)
    ns = splits or _lib.attn_auto_splits(B, Sq, HQ, HKV, cap, n_blk)
    wsb = _lib.attn_workspace_bytes(B, Sq, HQ, ns)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV) if wsb > 0 else None
    out = torch.full_like(q, 7.0)
    torch.ops.fdl.block_attn(q, k, v, lens.to(DEV), kb, vb, None, 0, D ** -0.5, out, ws, ns)
    for b in range(0, B, 5):
        L = int(lens[b])
        ref = O.block_attention(q[b:b + 1].float().cpu().numpy(), k[b:b + 1, :max(L, 1)].float().cpu().numpy(),
                                v[b:b + 1, :max(L, 1)].float().cpu().numpy(), [L],
                                k_blk=None if kb is None else kb[b:b + 1].float().cpu().numpy(),
                                v_blk=None if vb is None else vb[b:b + 1].float().cpu().numpy())
        assert_close(f"persistent Sq={Sq} blk={n_blk} splits={ns} b={b} L={L}", out[b:b + 1].float().cpu().numpy(),
                     ref, ATOL, RTOL)
