"""Golden end-to-end decode data from the REFERENCE's dKV sampler
(generation_functions.py:2132-2340, ``batch_sample_dkv``) on a tiny seeded
random-init model, run on CPU.

Usage:  python tests/golden/make_golden_decode.py [/path/to/reference]

The fixture stores the model geometry, the weight seed, the prompt, the
reference's generated tokens (bf16 and fp32 runs) and a teacher-forcing trace
of every forward the bf16 sampler ran (input tokens, kind, fed indices,
argmax / max probability / top-2 logit gap per position).  The weights are
regenerated from the seed by
``fast_v2_b200.block_decode.BlockDiffusionLM(init_device="cpu")`` (CPU
``torch.randn`` with a fixed generator), so the GPU test rebuilds the same
model without shipping a checkpoint.  The reference needs these local shims on
transformers 5.x, none of them copied from transformers: a stub
``configuration`` module (``bd_size``), a ``"default"`` RoPE init
(1/theta^(2i/d)), and list-style ``DynamicCache`` indexing / ``key_cache`` /
``value_cache`` views.
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
ROOT = HERE.parents[1]
if len(sys.argv) < 2 and "FV2_REFERENCE" not in os.environ:
    raise SystemExit("usage: python %s <path to the reference checkout> (or set FV2_REFERENCE)" % sys.argv[0])
REF = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["FV2_REFERENCE"])
MODELING = REF / "models/models--Efficient-Large-Model--Fast_dLLM_v2_7B/snapshots/0661abf5f9f0ee338970d091052a26c8efa51974/modeling.py"

# Tiny geometry with the 7B's GQA factor (7 query heads per KV head), D = 128.
GEO = dict(layers=2, hidden=896, heads=7, kv_heads=1, head_dim=128, ffn=1024, vocab=1024)
SEED = 1234
INIT_STD = 0.05
MASK_ID, STOP_ID, PAD_ID = 1023, 1022, 1021
B, PROMPT, GEN = 2, 64, 96


class _LayerView:
    """list-like key_cache / value_cache over a transformers-5 DynamicCache."""

    def __init__(self, cache, attr):
        self.cache, self.attr = cache, attr

    def __getitem__(self, i):
        return getattr(self.cache.layers[i], self.attr)

    def __setitem__(self, i, v):
        setattr(self.cache.layers[i], self.attr, v)

    def __len__(self):
        return len(self.cache.layers)


def install_shims():
    from transformers import Qwen2Config
    from transformers.cache_utils import DynamicCache
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    def _default_rope(config, device=None, *args, **kwargs):
        base = getattr(config, "rope_theta", None)
        if base is None:
            base = (getattr(config, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
        dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).float().to(device) / dim))
        return inv, 1.0

    ROPE_INIT_FUNCTIONS.setdefault("default", _default_rope)
    if not hasattr(DynamicCache, "__getitem__"):
        DynamicCache.__getitem__ = lambda self, i: (self.layers[i].keys, self.layers[i].values)
    if not hasattr(DynamicCache, "key_cache"):
        DynamicCache.key_cache = property(lambda self: _LayerView(self, "keys"))
        DynamicCache.value_cache = property(lambda self: _LayerView(self, "values"))

    pkg = types.ModuleType("fdllm_ref_pkg")
    pkg.__path__ = [str(MODELING.parent)]
    sys.modules["fdllm_ref_pkg"] = pkg
    cfg = types.ModuleType("fdllm_ref_pkg.configuration")

    class Fast_dLLM_QwenConfig(Qwen2Config):
        model_type = "fast_dllm_qwen_stub"

        def __init__(self, bd_size=32, **kw):
            self.bd_size = bd_size
            super().__init__(**kw)

    cfg.Fast_dLLM_QwenConfig = Fast_dLLM_QwenConfig
    sys.modules["fdllm_ref_pkg.configuration"] = cfg
    return Fast_dLLM_QwenConfig


def load_reference():
    sys.path.insert(0, str(REF))
    cfg_cls = install_shims()
    spec = importlib.util.spec_from_file_location("fdllm_ref_pkg.modeling", MODELING)
    modeling = importlib.util.module_from_spec(spec)
    sys.modules["fdllm_ref_pkg.modeling"] = modeling
    spec.loader.exec_module(modeling)
    import generation_functions as gf

    return modeling, gf, cfg_cls


def build_reference_model(modeling, cfg_cls, dtype):
    sys.path.insert(0, str(ROOT))
    from fast_v2_b200.block_decode import BlockDiffusionLM, Geometry

    geo = Geometry(**GEO, tie_embeddings=False)
    ours = BlockDiffusionLM(geo, device="cpu", dtype=dtype, seed=SEED, init_std=INIT_STD, init_device="cpu",
                            load_ops=False)
    cfg = cfg_cls(vocab_size=geo.vocab, hidden_size=geo.hidden, intermediate_size=geo.ffn,
                  num_hidden_layers=geo.layers, num_attention_heads=geo.heads, num_key_value_heads=geo.kv_heads,
                  max_position_embeddings=4096, rope_theta=geo.rope_theta, rms_norm_eps=geo.eps,
                  tie_word_embeddings=False, bd_size=32, attn_implementation="sdpa")
    model = modeling.Fast_dLLM_QwenForCausalLM(cfg).to(dtype).eval()
    # The rotary inverse frequencies stay fp32, as from_pretrained(torch_dtype=
    # bfloat16) leaves them (computed in fp32 at init, not in the checkpoint);
    # model.to(dtype) above would have rounded the buffer to bf16.
    rot = model.model.rotary_emb
    rot.inv_freq = 1.0 / (geo.rope_theta ** (torch.arange(0, geo.head_dim, 2, dtype=torch.int64).float()
                                             / geo.head_dim))
    q_out, kv_out = geo.heads * geo.head_dim, geo.kv_heads * geo.head_dim
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(ours.embed)
        model.lm_head.weight.copy_(ours.lm_head)
        model.model.norm.weight.copy_(ours.norm)
        for layer, w in zip(model.model.layers, ours.layers):
            a = layer.self_attn
            a.q_proj.weight.copy_(w["wqkv"][:q_out])
            a.k_proj.weight.copy_(w["wqkv"][q_out:q_out + kv_out])
            a.v_proj.weight.copy_(w["wqkv"][q_out + kv_out:])
            a.q_proj.bias.copy_(w["bqkv"][:q_out])
            a.k_proj.bias.copy_(w["bqkv"][q_out:q_out + kv_out])
            a.v_proj.bias.copy_(w["bqkv"][q_out + kv_out:])
            a.o_proj.weight.copy_(w["wo"])
            layer.mlp.gate_proj.weight.copy_(w["wgu"][:geo.ffn])
            layer.mlp.up_proj.weight.copy_(w["wgu"][geo.ffn:])
            layer.mlp.down_proj.weight.copy_(w["wd"])
            layer.input_layernorm.weight.copy_(w["ln1"])
            layer.post_attention_layernorm.weight.copy_(w["ln2"])
    return model


def run(dtype, record=False):
    """Free-running reference decode; with record=True also log every forward of
    the sampler: its input tokens, its kind (0 prefill/commit, 1 full dKV
    step, 2 cached dKV step), the fed indices, and the argmax / max
    probability of the (unshifted) logits per position as the sampler
    computes them (softmax in the model dtype), plus the top-2 logit gap."""
    modeling, gf, cfg_cls = load_reference()
    model = build_reference_model(modeling, cfg_cls, dtype)
    g = torch.Generator().manual_seed(SEED + 1)
    prompt = torch.randint(0, 1000, (B, PROMPT), generator=g)
    trace = []
    if record:
        fwd, fwd_dkv = model.forward, model.forward_dkv

        def _probe(kind, ids, fed, out):
            lg = out.logits
            p = torch.softmax(lg, dim=-1)
            top2 = lg.float().topk(2, dim=-1).values
            trace.append(dict(kind=kind, ids=ids.clone(), fed=None if fed is None else fed.clone(),
                              argmax=p.argmax(-1), pmax=p.max(-1).values.float(),
                              gap=(top2[..., 0] - top2[..., 1])))

        def forward(*a, **k):
            out = fwd(*a, **k)
            _probe(0, k["input_ids"], None, out)
            return out

        def forward_dkv(*a, **k):
            out = fwd_dkv(*a, **k)
            _probe(1 if k.get("is_full_step", True) else 2, k["input_ids"], k.get("fed_indices"), out)
            return out

        model.forward, model.forward_dkv = forward, forward_dkv
    sampler = types.MethodType(gf.Fast_dLLM_QwenForCausalLM.batch_sample_dkv, model)
    tok = types.SimpleNamespace(pad_token_id=PAD_ID)
    with torch.no_grad():
        res = sampler(prompt.clone(), tok, block_size=32, max_new_tokens=GEN, small_block_size=8, min_len=PROMPT,
                      seq_len=torch.full((B,), PROMPT, dtype=torch.long), mask_id=MASK_ID, threshold=0.9,
                      stop_token=STOP_ID, temperature=0.0)
    out = torch.stack([res[i] for i in range(B)])
    return prompt, out, trace


def replay_trace(dtype, trace):
    """Teacher-forced replay of a recorded sampler trace through the reference
    model in `dtype`: the same forwards in the same order, with the cache
    objects the sampler would hold (DynamicCache across blocks, a fresh
    DynamicBlockKV per block).  Returns (argmax, top logit) per record."""
    from transformers.cache_utils import DynamicCache

    modeling, gf, cfg_cls = load_reference()
    from utils.dynamic_block_kv import DynamicBlockKV

    model = build_reference_model(modeling, cfg_cls, dtype)
    pkv, block_kv, res = None, None, []
    with torch.no_grad():
        for t in trace:
            if t["kind"] == 0:
                out = model.forward(input_ids=t["ids"], use_cache=True, past_key_values=pkv,
                                    update_past_key_values=True, block_size=32)
                pkv, block_kv = out.past_key_values, None
            else:
                if pkv is None:
                    pkv = DynamicCache()
                if block_kv is None:
                    block_kv = DynamicBlockKV(0, GEO["layers"], B, GEO["kv_heads"], 32, GEO["head_dim"], dtype,
                                              torch.device("cpu"))
                out = model.forward_dkv(input_ids=t["ids"], use_cache=True, past_key_values=pkv,
                                        dkv_store=block_kv, fed_indices=t["fed"], is_full_step=t["kind"] == 1)
            lg = out.logits
            res.append((torch.softmax(lg, dim=-1).argmax(-1).numpy(), lg.float().max(-1).values.numpy()))
    return res


def gated_agreement(trace, replay, ulps=2.0):
    """Fraction of positions whose argmax equals the trace's, over positions
    whose top-2 logit gap exceeds `ulps` bf16 ulps of the top logit."""
    ok = n = ok_all = n_all = 0
    for t, (am, top) in zip(trace, replay):
        ref, gap = t["argmax"].numpy(), t["gap"].numpy()
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(top), 1e-30))) - 7)
        gate = gap > ulps * ulp
        ok += int(((am == ref) & gate).sum())
        n += int(gate.sum())
        ok_all += int((am == ref).sum())
        n_all += am.size
    return ok / max(1, n), ok_all / max(1, n_all)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    os.environ.setdefault("FAST_DLLM_DKV_REFRESH_STEPS", "4")
    prompt, out_bf16, trace = run(torch.bfloat16, record=True)
    _, out_f32, _ = run(torch.float32)
    agree = (out_bf16[:, PROMPT:] == out_f32[:, PROMPT:]).float().mean().item()
    tf_gated, tf_all = gated_agreement(trace, replay_trace(torch.float32, trace))
    rec = {}
    for i, t in enumerate(trace):
        rec[f"t{i}_kind"] = np.int64(t["kind"])
        rec[f"t{i}_ids"] = t["ids"].numpy()
        if t["fed"] is not None:
            rec[f"t{i}_fed"] = t["fed"].numpy()
        rec[f"t{i}_argmax"] = t["argmax"].numpy().astype(np.int32)
        rec[f"t{i}_pmax"] = t["pmax"].numpy().astype(np.float32)
        rec[f"t{i}_gap"] = t["gap"].numpy().astype(np.float32)
    np.savez_compressed(HERE / "decode_dkv.npz", prompt=prompt.numpy(), tokens_bf16=out_bf16.numpy(),
                        tokens_f32=out_f32.numpy(), seed=np.int64(SEED), init_std=np.float64(INIT_STD),
                        geo=np.array([GEO[k] for k in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn",
                                                       "vocab")]),
                        ids_special=np.array([MASK_ID, STOP_ID, PAD_ID]), refresh=np.int64(4),
                        n_trace=np.int64(len(trace)), ref_bf16_vs_f32_gen_agreement=np.float64(agree),
                        ref_tf_f32_agree_gated=np.float64(tf_gated), ref_tf_f32_agree_all=np.float64(tf_all), **rec)
    kinds = [t["kind"] for t in trace]
    print("tokens", tuple(out_bf16.shape), "trace", len(trace), "kinds", {k: kinds.count(k) for k in set(kinds)},
          "generated-token agreement bf16 vs fp32 reference", f"{agree:.4f}",
          f"teacher-forced fp32-vs-bf16 reference argmax agreement: gated {tf_gated:.4f} all {tf_all:.4f}")


if __name__ == "__main__":
    main()
