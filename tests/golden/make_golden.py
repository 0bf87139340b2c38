"""Generate the golden fixtures in this directory by running the REFERENCE's own
Python code (navneet-13/fast_v2) on CPU.

Usage:  python tests/golden/make_golden.py [/path/to/reference]

The reference is imported read-only.  Its modeling.py needs three small shims
on transformers 5.x (a stub ``configuration`` module with ``bd_size``, and
nothing else for the functions used here); they are defined below and touch
nothing but this process.  Each fixture stores the seeded inputs and the
reference outputs; tests/test_oracle_golden.py pins the CPU oracle to them and
the GPU parity tests compare the CUDA path with them.  Only this script reads
the reference; the fixtures travel, the reference does not.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if len(sys.argv) < 2 and "FV2_REFERENCE" not in os.environ:
    raise SystemExit("usage: python %s <path to the reference checkout> (or set FV2_REFERENCE)" % sys.argv[0])
REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["FV2_REFERENCE"])
MODELING = REF / "models/models--Efficient-Large-Model--Fast_dLLM_v2_7B/snapshots/0661abf5f9f0ee338970d091052a26c8efa51974/modeling.py"


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def load_reference():
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(REF / "cuda_bench"))
    pkg = types.ModuleType("fdllm_ref_pkg")
    pkg.__path__ = [str(MODELING.parent)]
    sys.modules["fdllm_ref_pkg"] = pkg
    from transformers import Qwen2Config

    cfg = types.ModuleType("fdllm_ref_pkg.configuration")

    class Fast_dLLM_QwenConfig(Qwen2Config):  # modeling.py:28 imports this name
        model_type = "fast_dllm_qwen_stub"

        def __init__(self, bd_size=32, **kw):
            self.bd_size = bd_size
            super().__init__(**kw)

    cfg.Fast_dLLM_QwenConfig = Fast_dLLM_QwenConfig
    sys.modules["fdllm_ref_pkg.configuration"] = cfg
    spec = importlib.util.spec_from_file_location("fdllm_ref_pkg.modeling", MODELING)
    modeling = importlib.util.module_from_spec(spec)
    sys.modules["fdllm_ref_pkg.modeling"] = modeling
    spec.loader.exec_module(modeling)
    import utils.attention_backends as ab
    import utils.block_sparse_cache as bsc
    import utils.dynamic_block_kv as dbk
    import utils.static_kv_cache as skv
    import test_correctness as tc

    return types.SimpleNamespace(modeling=modeling, skv=skv, dbk=dbk, bsc=bsc, ab=ab, tc=tc)


def gen_static_kv(ref):
    """StaticKVCache: prefill update (ragged 40), commit update (32), scratch write
    at kv_write_start, write_sparse with a repeated position."""
    g = torch.Generator().manual_seed(0)
    B, S, L, H, D = 2, 96, 2, 2, 64
    c = ref.skv.StaticKVCache(B, S, L, H, D, torch.bfloat16, torch.device("cpu"))
    out = {}
    rnd = lambda *shape: torch.randn(*shape, generator=g).to(torch.bfloat16)  # noqa: E731
    for step, s_len in (("pre", 40), ("commit", 32)):
        for l in range(L):
            k, v = rnd(B, s_len, H, D), rnd(B, s_len, H, D)
            out[f"{step}_k{l}"], out[f"{step}_v{l}"] = bits(k), bits(v)
            c.update(k, v, l)
    out["seq_len_after_commit"] = np.int64(c.get_seq_length())
    out["cache_seqlens"] = c.cache_seqlens.numpy().copy()
    c.set_kv_write_start(c.get_seq_length())
    c.set_scratch_seqlens(c.get_seq_length() + 16)
    c.prepare_write_idx(16)
    for l in range(L):
        k, v = rnd(B, 16, H, D), rnd(B, 16, H, D)
        out[f"scratch_k{l}"], out[f"scratch_v{l}"] = bits(k), bits(v)
        c.write_scratch_compiled(k, v, l)
    pos = torch.tensor([[3, 50, 51, 90, 7], [10, 11, 10, 95, 0]], dtype=torch.int64)
    out["sparse_pos"] = pos.numpy()
    for l in range(L):
        k, v = rnd(B, 5, H, D), rnd(B, 5, H, D)
        out[f"sparse_k{l}"], out[f"sparse_v{l}"] = bits(k), bits(v)
        c.write_sparse(k, v, l, pos)
    for l in range(L):
        out[f"final_k{l}"], out[f"final_v{l}"] = bits(c.key_cache[l]), bits(c.value_cache[l])
    out["scratch_seqlens"] = c.scratch_seqlens.numpy().copy()
    np.savez_compressed(HERE / "static_kv.npz", **out)


def gen_dynamic_block(ref):
    """DynamicBlockKV write_full + scatter with _dkv_fed_indices padding
    (repeated first index), and BlockSparseCache scatter of hidden rows."""
    g = torch.Generator().manual_seed(1)
    B, H, blk, D, L = 2, 2, 32, 64, 2
    buf = ref.dbk.DynamicBlockKV(0, L, B, H, blk, D, torch.bfloat16, torch.device("cpu"))
    prv = torch.zeros(B, blk, dtype=torch.bool)
    prv[0, 2:30] = True
    prv[1, ::3] = True
    fed, n_fed = ref.modeling.Fast_dLLM_QwenForCausalLM._dkv_fed_indices(prv)
    out = {"prv": prv.numpy(), "fed": fed.numpy(), "n_fed": np.int64(n_fed)}
    for l in range(L):
        kf = torch.randn(B, H, blk, D, generator=g).to(torch.bfloat16)
        vf = torch.randn(B, H, blk, D, generator=g).to(torch.bfloat16)
        buf.write_full(l, kf, vf)
        ks = torch.randn(B, H, n_fed, D, generator=g).to(torch.bfloat16)
        vs = torch.randn(B, H, n_fed, D, generator=g).to(torch.bfloat16)
        buf.write(l, ks, vs, fed)
        gk, gv = buf.get(l)
        out.update({f"full_k{l}": bits(kf), f"full_v{l}": bits(vf), f"sel_k{l}": bits(ks), f"sel_v{l}": bits(vs),
                    f"final_k{l}": bits(gk), f"final_v{l}": bits(gv)})
    hid = 256
    bs = ref.bsc.BlockSparseCache(L, B, blk, hid, torch.bfloat16, torch.device("cpu"))
    base = torch.randn(B, blk, hid, generator=g).to(torch.bfloat16)
    bs.cache_attn_output(1, base)
    tok = torch.tensor([[0, 5, 31], [4, 4, 9]], dtype=torch.int64)
    vals = torch.randn(B, 3, hid, generator=g).to(torch.bfloat16)
    bs.scatter_attn_output(1, tok, vals)
    out.update({"bsc_base": bits(base), "bsc_tok": tok.numpy(), "bsc_vals": bits(vals),
                "bsc_final": bits(bs.get_attn_output(1))})
    np.savez_compressed(HERE / "dynamic_block.npz", **out)


def gen_rmsnorm(ref):
    """ref_gather_input_rmsnorm (cuda_bench/test_correctness.py:33-50) on the
    reference's own case grid (test_correctness.py:128-144), with a
    non-trivial weight; the H=3584 case is shortened to S=64 rows."""
    cases_bf16 = [(1, 64, 128, 7, 1e-6), (2, 128, 256, 16, 1e-5), (1, 64, 3584, 32, 1e-6), (2, 256, 512, 24, 1e-6)]
    cases_f32 = [(1, 32, 64, 5, 1e-6), (3, 48, 96, 11, 1e-6), (1, 128, 512, 40, 1e-6)]
    out = {}
    for tag, dt, cases in (("bf16", torch.bfloat16, cases_bf16), ("f32", torch.float32, cases_f32)):
        for i, (b, s, h, t, eps) in enumerate(cases):
            g = torch.Generator().manual_seed(100 + i)
            x = torch.randn(b, s, h, generator=g).to(dt)
            idx = torch.randint(0, s, (b, t), generator=g, dtype=torch.long)
            w = (1.0 + 0.1 * torch.randn(h, generator=g)).to(dt)
            gath, normed = ref.tc.ref_gather_input_rmsnorm(x, idx, w, eps)
            key = f"{tag}_{i}"
            conv = bits if dt == torch.bfloat16 else (lambda z: z.numpy())
            out.update({f"{key}_x": conv(x), f"{key}_idx": idx.numpy(), f"{key}_w": conv(w),
                        f"{key}_eps": np.float64(eps), f"{key}_gathered": conv(gath), f"{key}_normed": conv(normed)})
        out[f"{tag}_n"] = np.int64(len(cases))
    np.savez_compressed(HERE / "rmsnorm.npz", **out)


def gen_attention(ref):
    """flash_kvcache_attention semantics through the reference's SDPA backend
    (AttentionBackend._sdpa_attention, utils/attention_backends.py:362-383) with
    the per-batch seqused mask of StaticKVCache.get_seqused_mask_batched
    (utils/static_kv_cache.py:295-302), in fp32 on bf16-representable inputs;
    plus the dynamic path: repeat_kv + SDPA over cat(prefix, block) under
    eval_mask (modeling.py:202-211, 390-411, 585-593) with a prefix of 40."""
    out = {}
    g = torch.Generator().manual_seed(7)
    B, Sq, Hq, Hkv, D, S = 2, 32, 14, 2, 128, 160
    q = (torch.randn(B, Sq, Hq, D, generator=g) / D ** 0.5).to(torch.bfloat16)
    k = torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16)
    seqlens = torch.tensor([130, 69], dtype=torch.int32)
    cache = ref.skv.StaticKVCache(B, S, 1, Hkv, D, torch.float32, torch.device("cpu"))
    mask = cache.get_seqused_mask_batched(seqlens)
    be = ref.ab.AttentionBackend(ref.ab.AttentionBackend.SDPA, None)
    o = be._sdpa_attention(q.float().transpose(1, 2), k.float().transpose(1, 2), v.float().transpose(1, 2), mask,
                           D ** -0.5, False, 0.0).transpose(1, 2)
    out.update({"kv_q": bits(q), "kv_k": bits(k), "kv_v": bits(v), "kv_seqlens": seqlens.numpy(),
                "kv_out": o.contiguous().numpy()})
    # dynamic path: BHSD prefix of 40 + block of 32, block-causal eval_mask
    P, blk = 40, 32
    qd = (torch.randn(1, Hq, blk, D, generator=g) / D ** 0.5).to(torch.bfloat16)
    pk = torch.randn(1, Hkv, P, D, generator=g).to(torch.bfloat16)
    pv = torch.randn(1, Hkv, P, D, generator=g).to(torch.bfloat16)
    bk = torch.randn(1, Hkv, blk, D, generator=g).to(torch.bfloat16)
    bv = torch.randn(1, Hkv, blk, D, generator=g).to(torch.bfloat16)
    fk = torch.cat((pk, bk), dim=-2).float()
    fv = torch.cat((pv, bv), dim=-2).float()
    m = ref.modeling.Fast_dLLM_QwenModel.eval_mask(None, blk, blk, P)
    n_rep = Hq // Hkv
    od = torch.nn.functional.scaled_dot_product_attention(
        qd.float(), ref.modeling.repeat_kv(fk, n_rep), ref.modeling.repeat_kv(fv, n_rep), attn_mask=m,
        scale=D ** -0.5).transpose(1, 2)
    out.update({"dyn_q": bits(qd), "dyn_pk": bits(pk), "dyn_pv": bits(pv), "dyn_bk": bits(bk), "dyn_bv": bits(bv),
                "dyn_mask": m.numpy(), "dyn_out": od.contiguous().numpy(),
                "dyn_repeat_k": bits(ref.modeling.repeat_kv(torch.cat((pk, bk), dim=-2), n_rep))})
    np.savez_compressed(HERE / "attention.npz", **out)


def gen_index_ops(ref):
    """_dkv_fed_indices, _focus_update_frozen and eval_mask known answers."""
    g = torch.Generator().manual_seed(11)
    M = ref.modeling.Fast_dLLM_QwenForCausalLM
    out = {}
    for i in range(6):
        prv = torch.rand(4, 32, generator=g) < (0.15 * i)
        fed, n = M._dkv_fed_indices(prv)
        out[f"fed_prv_{i}"], out[f"fed_idx_{i}"], out[f"fed_n_{i}"] = prv.numpy(), fed.numpy(), np.int64(n)
        mask = torch.rand(4, 32, generator=g) < 0.5
        frozen = torch.rand(4, 32, generator=g) < 0.2
        out[f"frz_mask_{i}"], out[f"frz_in_{i}"] = mask.numpy(), frozen.numpy()
        out[f"frz_out_{i}"] = M._focus_update_frozen(frozen, mask).numpy()
    for cl in (0, 40, 64):
        out[f"eval_mask_{cl}"] = ref.modeling.Fast_dLLM_QwenModel.eval_mask(None, 32, 32, cl).numpy()
    np.savez_compressed(HERE / "index_ops.npz", **out)


def gen_compaction(ref):
    """compact_batch of StaticKVCache, StaticBlockCache, DynamicBlockKV and
    BlockSparseCache (utils/static_kv_cache.py:350-398, :473-491,
    utils/dynamic_block_kv.py:52-56, utils/block_sparse_cache.py:141-147),
    applied twice (5 -> 3 -> 2 slots), then StaticKVCache.restore_full_batch."""
    g = torch.Generator().manual_seed(13)
    B, S, L, H, D, blk, hid = 5, 48, 2, 2, 64, 8, 64
    rnd = lambda *shape: torch.randn(*shape, generator=g).to(torch.bfloat16)  # noqa: E731
    steps = (torch.tensor([1, 2, 4]), torch.tensor([0, 2]))
    out = {"active_0": steps[0].numpy(), "active_1": steps[1].numpy()}
    c = ref.skv.StaticKVCache(B, S, L, H, D, torch.bfloat16, torch.device("cpu"))
    sb = ref.skv.StaticBlockCache(B, blk, L, H, D, torch.bfloat16, torch.device("cpu"))
    dk = ref.dbk.DynamicBlockKV(1, L + 1, B, H, blk, D, torch.bfloat16, torch.device("cpu"))
    bs = ref.bsc.BlockSparseCache(L, B, blk, hid, torch.bfloat16, torch.device("cpu"))
    for l in range(L):
        c.key_cache[l].copy_(rnd(B, S, H, D))
        c.value_cache[l].copy_(rnd(B, S, H, D))
        sb.key_cache[l].copy_(rnd(B, blk, H, D))
        sb.value_cache[l].copy_(rnd(B, blk, H, D))
    for l in dk.k:
        dk.k[l].copy_(rnd(B, H, blk, D))
        dk.v[l].copy_(rnd(B, H, blk, D))
    for name in ("layer_input", "attn_output", "mlp_input", "mlp_output"):
        getattr(bs, name).copy_(rnd(L, B, blk, hid))
    c.cache_seqlens.copy_(torch.tensor([40, 7, 33, 12, 25], dtype=torch.int32))
    c.scratch_seqlens.copy_(torch.tensor([41, 8, 34, 13, 26], dtype=torch.int32))

    def snapshot(tag):
        for l in range(L):
            out[f"{tag}_skv_k{l}"], out[f"{tag}_skv_v{l}"] = bits(c.key_cache[l]), bits(c.value_cache[l])
            out[f"{tag}_sbc_k{l}"], out[f"{tag}_sbc_v{l}"] = bits(sb.key_cache[l]), bits(sb.value_cache[l])
        for l in dk.k:
            out[f"{tag}_dbk_k{l}"], out[f"{tag}_dbk_v{l}"] = bits(dk.k[l]), bits(dk.v[l])
        for name in ("layer_input", "attn_output", "mlp_input", "mlp_output"):
            out[f"{tag}_bsc_{name}"] = bits(getattr(bs, name))
        out[f"{tag}_cache_seqlens"] = c.cache_seqlens.numpy().copy()
        out[f"{tag}_scratch_seqlens"] = c.scratch_seqlens.numpy().copy()
        out[f"{tag}_batch"] = np.int64(c.batch_size)

    snapshot("init")
    for i, act in enumerate(steps):
        for obj in (c, sb, dk, bs):
            obj.compact_batch(act)
        snapshot(f"step{i}")
    c.restore_full_batch()
    out["restored_batch"] = np.int64(c.batch_size)
    out["restored_shape"] = np.asarray(c.key_cache[0].shape, np.int64)
    out["restored_all_zero"] = np.bool_(all(bool((t == 0).all()) for t in c.key_cache + c.value_cache) and
                                        bool((c.cache_seqlens == 0).all()))
    np.savez_compressed(HERE / "compaction.npz", **out)


def gen_select(ref):
    """Token selection feeding the sparse gathers, run through the reference's
    own code: _focus_importance (modeling.py:214-237), _focus_select
    (modeling.py:240-306) and the cosine top-k of the sparse forward
    (modeling.py:868-874), in bf16 and fp32.  torch.topk leaves the order of
    equal values open, so the inputs are built without ties where the choice
    matters: distinct deltas, frozen sets that never force frozen padding,
    cosine targets spaced well apart."""
    M = ref.modeling
    g = torch.Generator().manual_seed(17)
    out = {}
    for tag, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
        # importance: the 7B head ratio (7 query heads per KV head), one row with nothing masked
        B, Hkv, rep, S, D = 2, 2, 7, 32, 128
        q = (torch.randn(B, Hkv * rep, S, D, generator=g) * 2.0).to(dt)
        k = torch.randn(B, Hkv, S, D, generator=g).to(dt)
        mask = torch.rand(B, S, generator=g) < 0.6
        mask[1] = False
        imp = M._focus_importance(q, M.repeat_kv(k, rep), mask, D ** -0.5)
        conv = bits if dt == torch.bfloat16 else (lambda z: z.numpy())
        out.update({f"imp_{tag}_q": conv(q), f"imp_{tag}_k": conv(k), f"imp_{tag}_mask": mask.numpy(),
                    f"imp_{tag}_out": imp.float().numpy()})
        # selection: distinct deltas (multiples of 2^-6), masks from sparse to full
        n_sel = 0
        for i in range(16):
            Bs, S = 4, 32
            vals = (torch.randperm(401, generator=g)[: Bs * S] - 200).float() / 64.0
            delta = vals.reshape(Bs, S).to(dt)
            mask = torch.rand(Bs, S, generator=g) < (0.15 + 0.05 * i)
            frozen = None
            if i % 3 == 1:
                # the same number of frozen decoded slots in every row: no frozen padding
                frozen = torch.zeros(Bs, S, dtype=torch.bool)
                for b in range(Bs):
                    dec = torch.nonzero(~mask[b]).flatten()
                    frozen[b, dec[: min(2, dec.numel())]] = True
                if len({int(f.sum()) for f in frozen}) != 1:
                    frozen = None
            avg, alpha = 1.0 + (i % 5), 1.0 + 0.5 * (i % 3)
            ro = 0.75 if i % 7 == 6 else None
            idx, ksel = M._focus_select(delta, mask, avg, alpha, ro, frozen=frozen)
            pad = -np.ones((Bs, S), np.int64)
            pad[:, :ksel] = idx.numpy()
            key = f"sel_{tag}_{i}"
            out.update({f"{key}_delta": conv(delta), f"{key}_mask": mask.numpy(),
                        f"{key}_frozen": (frozen if frozen is not None else torch.zeros(Bs, S, dtype=torch.bool)).numpy(),
                        f"{key}_has_frozen": np.bool_(frozen is not None),
                        f"{key}_args": np.array([avg, alpha, np.nan if ro is None else ro]),
                        f"{key}_idx": pad, f"{key}_ksel": np.int64(ksel)})
            n_sel += 1
        out[f"sel_{tag}_n"] = np.int64(n_sel)
        # cosine top-k: per-token target similarities spaced 1/40 apart
        B, S, H = 2, 32, 1024
        x = torch.randn(B, S, H, generator=g)
        z = torch.randn(B, S, H, generator=g)
        xh = x / x.norm(dim=-1, keepdim=True)
        z = z - (z * xh).sum(-1, keepdim=True) * xh
        zh = z / z.norm(dim=-1, keepdim=True)
        tgt = torch.stack([torch.randperm(S, generator=g) for _ in range(B)]).float() / 40.0 + 0.1
        y = (tgt[..., None] * xh + (1 - tgt[..., None] ** 2).sqrt() * zh) * (1.0 + torch.rand(B, S, 1, generator=g))
        hidden, cached = (x * 0.7).to(dt), y.to(dt)
        cos = torch.nn.functional.cosine_similarity(hidden, cached, dim=-1)
        n = int(0.25 * S)
        sel = cos.topk(n, dim=-1, largest=False).indices.sort(dim=-1).values
        out.update({f"cos_{tag}_hidden": conv(hidden), f"cos_{tag}_cached": conv(cached), f"cos_{tag}_n": np.int64(n),
                    f"cos_{tag}_cos": cos.float().numpy(), f"cos_{tag}_idx": sel.numpy()})
    np.savez_compressed(HERE / "select.npz", **out)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = load_reference()
    gen_static_kv(ref)
    gen_dynamic_block(ref)
    gen_rmsnorm(ref)
    gen_attention(ref)
    gen_index_ops(ref)
    gen_compaction(ref)
    gen_select(ref)
    for p in sorted(HERE.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
