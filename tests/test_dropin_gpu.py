"""The drop-in classes (reference API: StaticKVCache, StaticBlockCache,
DynamicBlockKV, BlockSparseCache, AttentionBackend, fused_sparse_extension)
driven the way the reference drives them, checked against the reference's
golden outputs and the CPU oracle."""
import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib
from fast_v2_b200.cuda_bench import fused_sparse_extension as fse
from fast_v2_b200.utils import (AttentionBackend, BlockSparseCache, DynamicBlockKV, StaticBlockCache, StaticKVCache,
                                get_attention_backend, patch_attention_layers, unpatch_attention_layers)
from oracle import kvcache_oracle as O
from tests._util import assert_close, bits_of, golden, t_from_bits

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(autouse=True)
def _clean():
    _lib.ensure_ops()
    _lib.last_device_error()
    yield
    assert _lib.last_device_error()[0] == 0


def test_static_kv_cache_reference_sequence():
    """update (prefill 40) -> update (commit 32) -> scratch write at
    kv_write_start -> write_sparse with a repeated position: identical bytes to
    the reference's StaticKVCache on CPU."""
    g = golden("static_kv")
    B, S, H, D = g["final_k0"].shape
    c = StaticKVCache(B, S, 2, H, D, torch.bfloat16, DEV)
    for step in ("pre", "commit"):
        for l in range(2):
            c.update(t_from_bits(g[f"{step}_k{l}"], DEV), t_from_bits(g[f"{step}_v{l}"], DEV), l)
    assert c.get_seq_length() == int(g["seq_len_after_commit"])
    assert np.array_equal(c.cache_seqlens.cpu().numpy(), g["cache_seqlens"])
    c.set_kv_write_start(c.get_seq_length())
    c.set_scratch_seqlens(c.get_seq_length() + 16)
    c.prepare_write_idx(16)
    for l in range(2):
        c.write_scratch_compiled(t_from_bits(g[f"scratch_k{l}"], DEV), t_from_bits(g[f"scratch_v{l}"], DEV), l)
    pos = torch.from_numpy(g["sparse_pos"]).to(DEV)
    for l in range(2):
        c.write_sparse(t_from_bits(g[f"sparse_k{l}"], DEV), t_from_bits(g[f"sparse_v{l}"], DEV), l, pos)
    for l in range(2):
        assert np.array_equal(bits_of(c.key_cache[l]), g[f"final_k{l}"])
        assert np.array_equal(bits_of(c.value_cache[l]), g[f"final_v{l}"])
    assert np.array_equal(c.scratch_seqlens.cpu().numpy(), g["scratch_seqlens"])
    k0, _ = c[0]
    assert k0.shape[1] == 72 and len(c) == 2


def test_static_kv_cache_per_sequence_append_and_compaction():
    B, S, H, D = 4, 128, 4, 128
    c = StaticKVCache(B, S, 3, H, D, torch.bfloat16, DEV)
    lens = torch.tensor([0, 32, 96, 7], dtype=torch.int32, device=DEV)
    ks = [torch.randn(B, 32, H, D, device=DEV).to(torch.bfloat16) for _ in range(3)]
    vs = [torch.randn(B, 32, H, D, device=DEV).to(torch.bfloat16) for _ in range(3)]
    c.append_layers(ks, vs, lens)
    for l in range(3):
        for b in range(B):
            s = int(lens[b])
            assert torch.equal(c.key_cache[l][b, s:s + 32], ks[l][b])
            assert torch.equal(c.value_cache[l][b, s:s + 32], vs[l][b])
    keep = torch.tensor([3, 1], device=DEV)
    before = c.key_cache[2][keep].clone()
    c.compact_batch(keep)
    assert c.batch_size == 2 and torch.equal(c.key_cache[2], before)


def test_static_block_cache_update_and_reset():
    B, blk, H, D = 2, 32, 4, 128
    sb = StaticBlockCache(B, blk, 2, H, D, torch.bfloat16, DEV)
    k = torch.randn(B, blk, H, D, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, blk, H, D, device=DEV).to(torch.bfloat16)
    kk, vv = sb.update(k, v, 1)
    assert torch.equal(kk, k) and torch.equal(vv, v) and len(sb) == 2 and sb.get_seq_length() == blk
    sb.reset()
    assert len(sb) == 0


def test_dynamic_block_kv_reference_sequence():
    g = golden("dynamic_block")
    B, H, blk, D = g["full_k0"].shape
    buf = DynamicBlockKV(0, 2, B, H, blk, D, torch.bfloat16, DEV)
    fed = torch.from_numpy(g["fed"]).to(DEV)
    for l in range(2):
        buf.write_full(l, t_from_bits(g[f"full_k{l}"], DEV), t_from_bits(g[f"full_v{l}"], DEV))
        buf.write(l, t_from_bits(g[f"sel_k{l}"], DEV), t_from_bits(g[f"sel_v{l}"], DEV), fed)
        k, v = buf.get(l)
        assert np.array_equal(bits_of(k), g[f"final_k{l}"]) and np.array_equal(bits_of(v), g[f"final_v{l}"])


def test_dynamic_block_kv_reference_known_answers():
    """tests/test_dkv.py:54-69 and tests/test_focus.py:611-636 of the reference
    (there in fp32 on CPU; here in bf16 on the GPU)."""
    B, Hkv, block, D, L = 1, 4, 8, 16, 28
    buf = DynamicBlockKV(0, L, B, Hkv, block, D, torch.bfloat16, DEV)
    assert set(buf.k.keys()) == set(range(L))
    k0 = (torch.arange(B * Hkv * block * D) % 251).reshape(B, Hkv, block, D).to(torch.bfloat16).to(DEV)
    buf.write_full(0, k0, k0.clone())
    buf.write(0, torch.zeros(B, Hkv, 2, D, dtype=torch.bfloat16, device=DEV),
              torch.zeros(B, Hkv, 2, D, dtype=torch.bfloat16, device=DEV), torch.tensor([[2, 5]], device=DEV))
    gk, _ = buf.get(0)
    assert torch.equal(gk[:, :, 2], torch.zeros_like(gk[:, :, 2])) and torch.equal(gk[:, :, 3], k0[:, :, 3])
    buf2 = DynamicBlockKV(2, 3, 1, 2, 5, 8, torch.bfloat16, DEV)
    buf2.write_full(2, torch.zeros(1, 2, 5, 8, dtype=torch.bfloat16, device=DEV),
                    torch.zeros(1, 2, 5, 8, dtype=torch.bfloat16, device=DEV))
    buf2.write(2, torch.ones(1, 2, 2, 8, dtype=torch.bfloat16, device=DEV),
               2 * torch.ones(1, 2, 2, 8, dtype=torch.bfloat16, device=DEV), torch.tensor([[1, 3]], device=DEV))
    gk, gv = buf2.get(2)
    assert gk[0, 0, 1, 0] == 1 and gk[0, 0, 3, 0] == 1 and gk[0, 0, 0, 0] == 0 and gk[0, 0, 2, 0] == 0
    assert gv[0, 0, 1, 0] == 2 and gv[0, 0, 0, 0] == 0


def test_block_sparse_cache_scatter_reference():
    g = golden("dynamic_block")
    B, blk, hid = g["bsc_base"].shape
    bs = BlockSparseCache(2, B, blk, hid, torch.bfloat16, DEV)
    bs.cache_attn_output(1, t_from_bits(g["bsc_base"], DEV))
    bs.scatter_attn_output(1, torch.from_numpy(g["bsc_tok"]).to(DEV), t_from_bits(g["bsc_vals"], DEV))
    assert np.array_equal(bits_of(bs.get_attn_output(1)), g["bsc_final"])
    bs.cache_mlp_output(0, t_from_bits(g["bsc_base"], DEV))
    bs.scatter_mlp_output(0, torch.from_numpy(g["bsc_tok"]).to(DEV), t_from_bits(g["bsc_vals"], DEV))
    assert np.array_equal(bits_of(bs.get_mlp_output(0)), g["bsc_final"])


def test_fused_sparse_extension_pair_and_ops_golden():
    g = golden("rmsnorm")

    class Norm(torch.nn.Module):
        def __init__(self, w, eps):
            super().__init__()
            self.weight = torch.nn.Parameter(w, requires_grad=False)
            self.variance_epsilon = eps

    for i in range(int(g["bf16_n"])):
        k = f"bf16_{i}"
        x = t_from_bits(g[f"{k}_x"], DEV)
        idx = torch.from_numpy(g[f"{k}_idx"]).to(DEV)
        gath, normed = fse.fused_gather_input_rmsnorm_pair(x, idx, Norm(t_from_bits(g[f"{k}_w"], DEV),
                                                                         float(g[f"{k}_eps"])))
        assert np.array_equal(bits_of(gath), g[f"{k}_gathered"])
        assert_close(k, normed.float().cpu().numpy(), O.bf16_to_f32(g[f"{k}_normed"]), ATOL, RTOL)
    assert fse.fused_gather_input_rmsnorm_pair(torch.zeros(1, 4, 8), torch.zeros(1, 2, dtype=torch.long),
                                               Norm(torch.ones(8), 1e-6)) is None
    ops = fse.get_fused_ops()
    for i in range(int(g["f32_n"])):
        k = f"f32_{i}"
        x = torch.from_numpy(g[f"{k}_x"]).to(DEV)
        idx = torch.from_numpy(g[f"{k}_idx"]).to(DEV)
        w = torch.from_numpy(g[f"{k}_w"]).to(DEV)
        eps = float(g[f"{k}_eps"])
        out = ops.gather_rmsnorm_cuda(x, idx, w, eps)
        assert_close(k, out.cpu().numpy(), g[f"{k}_normed"], 1e-5, 1e-5)
        gathered, pre = ops.fused_gather_input_rmsnorm_pair(x, idx, eps)
        assert np.array_equal(gathered.cpu().numpy(), g[f"{k}_gathered"])
        assert_close(k + "pre", (pre * w).cpu().numpy(), g[f"{k}_normed"], 1e-5, 1e-5)
    # scatter_and_return_cuda writes both targets
    cache = torch.zeros(2, 10, 16, device=DEV)
    hid = torch.zeros(2, 10, 16, device=DEV)
    vals = torch.randn(2, 3, 16, device=DEV)
    idx = torch.tensor([[1, 4, 9], [0, 2, 3]], device=DEV)
    r = ops.scatter_and_return_cuda(vals, idx, cache, hid)
    assert r is hid and torch.equal(cache[0, 4], vals[0, 1]) and torch.equal(hid[1, 3], vals[1, 2])


def test_attention_backend_flash_kvcache_golden():
    g = golden("attention")
    be = get_attention_backend("auto")
    assert isinstance(be, AttentionBackend) and be.name == "fdl_b200"
    be.plan_flashinfer()
    q, k, v = (t_from_bits(g[n], DEV) for n in ("kv_q", "kv_k", "kv_v"))
    out = be.flash_kvcache_attention(q, k, v, torch.from_numpy(g["kv_seqlens"]).to(DEV))
    assert_close("flash_kvcache", out.float().cpu().numpy(), g["kv_out"], ATOL, RTOL)


def test_attention_backend_block_attention_dynamic_golden():
    g = golden("attention")
    be = get_attention_backend()
    q = t_from_bits(g["dyn_q"], DEV).transpose(1, 2).contiguous()
    pk, pv = (t_from_bits(g[n], DEV).transpose(1, 2) for n in ("dyn_pk", "dyn_pv"))  # BHSD memory
    bk, bv = (t_from_bits(g[n], DEV).transpose(1, 2) for n in ("dyn_bk", "dyn_bv"))
    lens = torch.full((1,), pk.shape[1], dtype=torch.int32, device=DEV)
    out = be.block_attention(q, pk, pv, lens, bk, bv, mask_block=32)
    assert_close("dynamic", out.float().cpu().numpy(), g["dyn_out"], ATOL, RTOL)


class _TinyAttn(torch.nn.Module):
    def __init__(self, layer_idx, hidden=256, hq=4, hkv=2, d=64 * 2):
        super().__init__()
        self.layer_idx, self.head_dim, self.scaling = layer_idx, d, d ** -0.5
        self.q_proj = torch.nn.Linear(hidden, hq * d)
        self.k_proj = torch.nn.Linear(hidden, hkv * d)
        self.v_proj = torch.nn.Linear(hidden, hkv * d)
        self.o_proj = torch.nn.Linear(hq * d, hidden, bias=False)

    def forward(self, *a, **k):  # never reached when patched with a StaticKVCache
        raise AssertionError("unpatched forward called")


def test_patched_attention_forward_commit_and_scratch():
    torch.manual_seed(0)
    L, B, hidden, hq, hkv, d, S = 2, 2, 256, 4, 2, 128, 128

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.model = torch.nn.Module()
            self.model.layers = torch.nn.ModuleList()
            for i in range(L):
                layer = torch.nn.Module()
                layer.self_attn = _TinyAttn(i, hidden, hq, hkv, d)
                self.model.layers.append(layer)

    m = Model().to(DEV).to(torch.bfloat16).requires_grad_(False)
    be = get_attention_backend()
    orig = patch_attention_layers(m, be)
    cache = StaticKVCache(B, S, L, hkv, d, torch.bfloat16, DEV)
    x = torch.randn(B, 32, hidden, device=DEV).to(torch.bfloat16)
    cos = torch.ones(B, 32, d, device=DEV, dtype=torch.bfloat16)
    sin = torch.zeros(B, 32, d, device=DEV, dtype=torch.bfloat16)
    outs = [m.model.layers[l].self_attn.forward(x, (cos, sin), past_key_value=cache, update_past_key_values=True)
            for l in range(L)]
    assert cache.get_seq_length() == 32
    # reference semantics: attention over the 32 committed keys (scratch_seqlens = 32)
    for l in range(L):
        a = m.model.layers[l].self_attn
        q = a.q_proj(x).view(B, 32, hq, d)
        ref = O.block_attention(q.float().cpu().numpy(), cache.key_cache[l].float().cpu().numpy(),
                                cache.value_cache[l].float().cpu().numpy(), [32, 32])
        ctx = torch.from_numpy(ref).to(DEV).to(torch.bfloat16).reshape(B, 32, -1)
        assert_close(f"layer{l}", outs[l].float().cpu().numpy(), a.o_proj(ctx).float().cpu().numpy(), 5e-2, 5e-2)
    unpatch_attention_layers(m, orig)
    assert m.model.layers[0].self_attn.forward == orig[0]


def test_compaction_of_every_cache_matches_reference_in_place():
    """compact_batch twice (5 -> 3 -> 2 slots) on StaticKVCache,
    StaticBlockCache, DynamicBlockKV and BlockSparseCache: the same bytes as
    the reference's index_select compaction, with every buffer still at its
    original address; restore_full_batch grows the views back, zeroed."""
    g = golden("compaction")
    L, (B, S, H, D) = 2, g["init_skv_k0"].shape
    blk, hid = g["init_sbc_k0"].shape[1], g["init_bsc_layer_input"].shape[-1]
    c = StaticKVCache(B, S, L, H, D, torch.bfloat16, DEV)
    sb = StaticBlockCache(B, blk, L, H, D, torch.bfloat16, DEV)
    dk = DynamicBlockKV(1, L + 1, B, H, blk, D, torch.bfloat16, DEV)
    bs = BlockSparseCache(L, B, blk, hid, torch.bfloat16, DEV)
    for l in range(L):
        c.key_cache[l].copy_(t_from_bits(g[f"init_skv_k{l}"], DEV))
        c.value_cache[l].copy_(t_from_bits(g[f"init_skv_v{l}"], DEV))
        sb.key_cache[l].copy_(t_from_bits(g[f"init_sbc_k{l}"], DEV))
        sb.value_cache[l].copy_(t_from_bits(g[f"init_sbc_v{l}"], DEV))
    for l in dk.k:
        dk.k[l].copy_(t_from_bits(g[f"init_dbk_k{l}"], DEV))
        dk.v[l].copy_(t_from_bits(g[f"init_dbk_v{l}"], DEV))
    names = ("layer_input", "attn_output", "mlp_input", "mlp_output")
    for name in names:
        getattr(bs, name).copy_(t_from_bits(g[f"init_bsc_{name}"], DEV))
    c.cache_seqlens.copy_(torch.from_numpy(g["init_cache_seqlens"]))
    c.scratch_seqlens.copy_(torch.from_numpy(g["init_scratch_seqlens"]))

    def tensors():
        return (c.key_cache + c.value_cache + sb.key_cache + sb.value_cache + list(dk.k.values()) +
                list(dk.v.values()) + [getattr(bs, n) for n in names] + [c.cache_seqlens, c.scratch_seqlens])

    ptrs = [t.data_ptr() for t in tensors()]
    for i in range(2):
        act = torch.from_numpy(g[f"active_{i}"]).to(DEV)
        for obj in (c, sb, dk, bs):
            obj.compact_batch(act)
        tag = f"step{i}"
        for l in range(L):
            assert np.array_equal(bits_of(c.key_cache[l]), g[f"{tag}_skv_k{l}"])
            assert np.array_equal(bits_of(c.value_cache[l]), g[f"{tag}_skv_v{l}"])
            assert np.array_equal(bits_of(sb.key_cache[l]), g[f"{tag}_sbc_k{l}"])
            assert np.array_equal(bits_of(sb.value_cache[l]), g[f"{tag}_sbc_v{l}"])
        for l in dk.k:
            assert np.array_equal(bits_of(dk.k[l]), g[f"{tag}_dbk_k{l}"])
            assert np.array_equal(bits_of(dk.v[l]), g[f"{tag}_dbk_v{l}"])
        for name in names:
            assert np.array_equal(bits_of(getattr(bs, name)), g[f"{tag}_bsc_{name}"]), name
        assert np.array_equal(c.cache_seqlens.cpu().numpy(), g[f"{tag}_cache_seqlens"])
        assert np.array_equal(c.scratch_seqlens.cpu().numpy(), g[f"{tag}_scratch_seqlens"])
        assert c.batch_size == sb.batch_size == dk.batch_size == bs.batch_size == int(g[f"{tag}_batch"])
        assert [t.data_ptr() for t in tensors()] == ptrs
    c.restore_full_batch()
    assert c.batch_size == int(g["restored_batch"]) and list(c.key_cache[0].shape) == list(g["restored_shape"])
    assert all(int(t.abs().max()) == 0 for t in c.key_cache + c.value_cache + [c.cache_seqlens])
    assert [t.data_ptr() for t in c.key_cache + c.value_cache] == ptrs[:2 * L]


def test_compaction_at_decode_size_and_refused_orders():
    """A 16-slot cache of 2304 positions (the 7B geometry's KV heads) drops
    5 finished slots: equal to index_select.  A list outside i <= a[i] is
    refused: ValueError from the cache, and from the raw op nothing moves and
    the device status names the offending entry."""
    B, S, H, D, L = 16, 2304, 4, 128, 4
    c = StaticKVCache(B, S, L, H, D, torch.bfloat16, DEV)
    gen = torch.Generator(device=DEV).manual_seed(3)
    for t in c.key_cache + c.value_cache:
        t.copy_(torch.randn(t.shape, generator=gen, device=DEV).to(torch.bfloat16))
    c.cache_seqlens.copy_(torch.arange(B, dtype=torch.int32, device=DEV) * 100)
    act = torch.tensor([0, 2, 3, 6, 7, 8, 10, 11, 13, 14, 15], device=DEV)
    want = [t[act].clone() for t in c.key_cache + c.value_cache]
    c.compact_batch(act)
    for got, exp in zip(c.key_cache + c.value_cache, want):
        assert torch.equal(got, exp)
    assert torch.equal(c.cache_seqlens, act.to(torch.int32) * 100)
    with pytest.raises(ValueError):
        c.compact_batch(torch.tensor([1, 0], device=DEV))
    buf = torch.arange(4 * 8, dtype=torch.float32, device=DEV).reshape(4, 8)
    keep = buf.clone()
    torch.ops.fdl.kv_compact([buf], torch.tensor([1, 0], device=DEV))
    assert torch.equal(buf, keep)
    assert _lib.last_device_error() == (1, 0)  # FDL_DEV_INDEX, active[1] = 0 < 1


def test_seqused_masks_match_the_reference_semantics_and_attention():
    """get_seqused_mask / get_seqused_mask_batched (utils/static_kv_cache.py:
    286-302): an additive [B, 1, 1, max_S] mask, 0 for key j < the valid
    length and -inf beyond, written into one persistent buffer (the same
    tensor every call, so a captured graph sees the refill).  SDPA under the
    batched mask equals the library's flash_kvcache over the same lengths, as
    the reference's SDPA fallback relies on."""
    B, S, L, H, D = 3, 160, 1, 4, 128
    cache = StaticKVCache(B, S, L, H, D, torch.bfloat16, DEV)
    m1 = cache.get_seqused_mask(37)
    ref = np.zeros((B, 1, 1, S), np.float32)
    ref[..., 37:] = -np.inf
    assert m1.shape == (B, 1, 1, S) and np.array_equal(m1.float().cpu().numpy(), ref)
    seqused = torch.tensor([5, 160, 64], dtype=torch.int32, device=DEV)
    m2 = cache.get_seqused_mask_batched(seqused)
    assert m2.data_ptr() == m1.data_ptr()
    ref = np.zeros((B, 1, 1, S), np.float32)
    for b, n in enumerate([5, 160, 64]):
        ref[b, ..., n:] = -np.inf
    assert np.array_equal(m2.float().cpu().numpy(), ref)
    g = torch.Generator(device=DEV).manual_seed(3)
    q = (torch.randn(B, 32, H * 7, D, generator=g, device=DEV) / D ** 0.5).to(torch.bfloat16)
    k = torch.randn(B, S, H, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, S, H, D, generator=g, device=DEV).to(torch.bfloat16)
    kk = k.transpose(1, 2).repeat_interleave(7, dim=1).float()
    vv = v.transpose(1, 2).repeat_interleave(7, dim=1).float()
    sdpa = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2).float(), kk, vv,
                                                            attn_mask=m2.float()).transpose(1, 2)
    out = get_attention_backend().flash_kvcache_attention(q, k, v, seqused)
    assert_close("flash_kvcache vs SDPA under the seqused mask", out.float().cpu().numpy(),
                 sdpa.cpu().numpy(), ATOL, RTOL)
