"""Golden end-to-end decode data from the REFERENCE's static-cache sampler
(generation_functions.py:243-900, ``batch_sample_dynamo``, eager mode, no
block cache) on the tiny seeded random-init model of make_golden_decode.py,
run on CPU.

Usage:  python tests/golden/make_golden_static.py <path to the reference checkout>

The static sampler drives ``StaticKVCache`` (utils/static_kv_cache.py) and
the patched attention forward (utils/attention_backends.py:791-898): every
forward writes its K/V into the cache (the commit at the committed length
with ``update``, a diffusion step as scratch rows at ``kv_write_start`` with
``write_scratch_compiled``) and attends with ``flash_kvcache_attention`` over
``cache[:scratch_seqlens]`` with ``is_causal=False`` -- so the prompt prefill
is bidirectional over the whole prompt, unlike the dKV sampler's block-causal
prefill.  That attention call needs flash-attn or FlashInfer on a GPU; here
the reference's own backend object is given a CPU stand-in with the published
semantics of flash-attn's ``flash_attn_with_kvcache(q, k_cache, v_cache,
cache_seqlens=..., softmax_scale=..., causal=False)`` (flash-attn 2.x API):
query row i of sequence b attends keys [0, cache_seqlens[b]) of its KV head
(query head h reads KV head h // (Hq / Hkv)), softmax in fp32, output in the
query dtype.  Nothing else of the reference is changed.

The fixture stores the prompt, the sampler's generated tokens (bf16 and fp32
runs) and a trace of every forward of the bf16 run: kind 0 = prefill /
commit (``update_past_key_values=True``), kind 3 = diffusion step
(``forward_dynamo`` with scratch writes), the input tokens, and per position
the argmax / max probability of the unshifted logits (softmax in the model
dtype) and the top-2 logit gap.  The reference's own fp32 path replayed on
the same trace gives the noise floor.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if len(sys.argv) < 2 and "FV2_REFERENCE" not in os.environ:
    raise SystemExit("usage: python %s <path to the reference checkout> (or set FV2_REFERENCE)" % sys.argv[0])
os.environ.setdefault("FV2_REFERENCE", sys.argv[1] if len(sys.argv) > 1 else "")
sys.path.insert(0, str(HERE))
import make_golden_decode as base  # noqa: E402  (shares the model, shims and loader)

BLOCK = 32


def kvcache_attention_cpu(q, k_cache, v_cache, cache_seqlens=None, softmax_scale=None, causal=False):
    """flash_attn_with_kvcache semantics (causal=False) on CPU: BSHD q
    [B, Sq, Hq, D] over k/v_cache [B, S, Hkv, D], keys [0, cache_seqlens[b])."""
    assert not causal
    B, Sq, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    scale = softmax_scale if softmax_scale is not None else D ** -0.5
    out = torch.empty_like(q)
    for b in range(B):
        n = int(cache_seqlens[b])
        k = k_cache[b, :n].float().repeat_interleave(Hq // Hkv, dim=1)  # [n, Hq, D]
        v = v_cache[b, :n].float().repeat_interleave(Hq // Hkv, dim=1)
        s = torch.einsum("qhd,khd->hqk", q[b].float(), k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hqk,khd->qhd", p, v).to(q.dtype)
    return out


def install_kvcache_standin():
    from utils.attention_backends import get_attention_backend

    be = get_attention_backend(os.environ.get("FAST_DLLM_ATTENTION_BACKEND", "auto"))
    be.name = be.FLASH2
    be._impl = {"kvcache": kvcache_attention_cpu}
    be._kvcache_dispatch_logged = True
    return be


def _probe(trace, kind, ids, out):
    lg = out.logits
    p = torch.softmax(lg, dim=-1)
    top2 = lg.float().topk(2, dim=-1).values
    trace.append(dict(kind=kind, ids=ids.clone(), argmax=p.argmax(-1), pmax=p.max(-1).values.float(),
                      gap=(top2[..., 0] - top2[..., 1])))


def run(dtype, record=False):
    modeling, gf, cfg_cls = base.load_reference()
    install_kvcache_standin()
    model = base.build_reference_model(modeling, cfg_cls, dtype)
    g = torch.Generator().manual_seed(base.SEED + 1)
    prompt = torch.randint(0, 1000, (base.B, base.PROMPT), generator=g)
    trace = []
    if record:
        fwd, fwd_dyn = model.forward, model.forward_dynamo

        def forward(*a, **k):
            out = fwd(*a, **k)
            _probe(trace, 0, k["input_ids"], out)
            return out

        def forward_dynamo(*a, **k):
            out = fwd_dyn(*a, **k)
            _probe(trace, 3, k["input_ids"], out)
            return out

        model.forward, model.forward_dynamo = forward, forward_dynamo
    sampler = types.MethodType(gf.Fast_dLLM_QwenForCausalLM.batch_sample_dynamo, model)
    tok = types.SimpleNamespace(pad_token_id=base.PAD_ID)
    with torch.no_grad():
        res = sampler(prompt.clone(), tok, block_size=BLOCK, max_new_tokens=base.GEN, small_block_size=8,
                      min_len=base.PROMPT, seq_len=torch.full((base.B,), base.PROMPT, dtype=torch.long),
                      mask_id=base.MASK_ID, threshold=0.9, stop_token=base.STOP_ID, temperature=0.0)
    out = torch.stack([res[i] for i in range(base.B)])  # {slot: tokens} (BatchBucket.get_results)
    return prompt, out, trace


def replay_trace(dtype, trace):
    """Teacher-forced replay of the recorded forwards through the reference
    model in `dtype` with the sampler's own cache calls: a StaticKVCache, the
    patched attention layers, and at the first diffusion step of each block
    the per-block set-up of generation_functions.py:586-597."""
    modeling, gf, cfg_cls = base.load_reference()
    from utils.attention_backends import patch_attention_layers
    from utils.static_kv_cache import StaticKVCache

    be = install_kvcache_standin()
    model = base.build_reference_model(modeling, cfg_cls, dtype)
    patch_attention_layers(model, be, None)
    G = base.GEO
    cache = StaticKVCache(batch_size=base.B, max_seq_len=base.PROMPT + base.GEN + 2 * BLOCK, num_layers=G["layers"],
                          num_kv_heads=G["kv_heads"], head_dim=G["head_dim"], dtype=dtype,
                          device=torch.device("cpu"))
    res, prev = [], 0
    with torch.no_grad():
        for t in trace:
            if t["kind"] == 0:
                out = model.forward(input_ids=t["ids"], use_cache=True, past_key_values=cache,
                                    update_past_key_values=True, block_size=BLOCK)
            else:
                past_len = cache.get_seq_length()
                if prev == 0:
                    cache.set_kv_write_start(past_len)
                    cache.set_scratch_seqlens(past_len + BLOCK)
                    cache.prepare_write_idx(BLOCK)
                pos = torch.arange(past_len, past_len + BLOCK)
                out = model.forward_dynamo(input_ids=t["ids"], use_cache=True, past_key_values=cache,
                                           update_past_key_values=False, cache_position=pos,
                                           logits_to_keep=BLOCK)
            prev = t["kind"]
            lg = out.logits
            res.append((torch.softmax(lg, dim=-1).argmax(-1).numpy(), lg.float().max(-1).values.numpy()))
    return res


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    prompt, out_bf16, trace = run(torch.bfloat16, record=True)
    _, out_f32, _ = run(torch.float32)
    P = base.PROMPT
    n = min(out_bf16.shape[1], out_f32.shape[1])
    agree = (out_bf16[:, P:n] == out_f32[:, P:n]).float().mean().item()
    tf_gated, tf_all = base.gated_agreement(trace, replay_trace(torch.float32, trace))
    self_gated, _ = base.gated_agreement(trace, replay_trace(torch.bfloat16, trace))
    rec = {}
    for i, t in enumerate(trace):
        rec[f"t{i}_kind"] = np.int64(t["kind"])
        rec[f"t{i}_ids"] = t["ids"].numpy()
        rec[f"t{i}_argmax"] = t["argmax"].numpy().astype(np.int32)
        rec[f"t{i}_pmax"] = t["pmax"].numpy().astype(np.float32)
        rec[f"t{i}_gap"] = t["gap"].numpy().astype(np.float32)
    G = base.GEO
    np.savez_compressed(HERE / "decode_static.npz", prompt=prompt.numpy(), tokens_bf16=out_bf16.numpy(),
                        tokens_f32=out_f32.numpy(), seed=np.int64(base.SEED), init_std=np.float64(base.INIT_STD),
                        geo=np.array([G[k] for k in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn",
                                                     "vocab")]),
                        ids_special=np.array([base.MASK_ID, base.STOP_ID, base.PAD_ID]),
                        n_trace=np.int64(len(trace)), ref_bf16_vs_f32_gen_agreement=np.float64(agree),
                        ref_tf_f32_agree_gated=np.float64(tf_gated), ref_tf_f32_agree_all=np.float64(tf_all), **rec)
    kinds = [t["kind"] for t in trace]
    print("tokens", tuple(out_bf16.shape), "trace", len(trace), "kinds", {k: kinds.count(k) for k in set(kinds)},
          f"generated-token agreement bf16 vs fp32 reference {agree:.4f}",
          f"teacher-forced fp32-vs-bf16 reference argmax agreement: gated {tf_gated:.4f} all {tf_all:.4f}",
          f"bf16 replay vs recorded bf16 run (must be 1): {self_gated:.4f}")


if __name__ == "__main__":
    main()
