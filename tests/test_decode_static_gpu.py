"""End-to-end decode with the static-cache schedule vs the reference's own
static-cache sampler ``batch_sample_dynamo`` (tests/golden/decode_static.npz,
made by make_golden_static.py from generation_functions.py:243-900 on CPU in
bf16, eager mode, no block cache).

That sampler writes every forward's K/V into the committed cache (commit at
the committed length; each diffusion step as scratch rows at
``kv_write_start``) and attends over cache[:scratch_seqlens] with no mask --
the prompt prefill included.  The replay runs the same forwards with the same
input tokens through DecodeState.forward_commit(mask_block=0) and
DecodeState.forward_scratch; outside near ties our argmax must agree with the
reference's bf16 argmax at least as often (within 0.5 %) as the reference's
own fp32 path does.
"""
import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib
from fast_v2_b200.block_decode import BlockDiffusionDecoder, BlockDiffusionLM, Geometry
from tests._util import golden
from tests.test_decode_gpu import KV_STORE, NEAR_TIE_ULPS, _bf16_ulp

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _setup(gen=None, **kw):
    g = golden("decode_static")
    L, H, hq, hkv, d, ffn, V = (int(x) for x in g["geo"])
    model = BlockDiffusionLM(Geometry(L, H, hq, hkv, d, ffn, V), device=DEV, seed=int(g["seed"]),
                             init_std=float(g["init_std"]), init_device="cpu")
    mask_id, stop_id, pad_id = (int(x) for x in g["ids_special"])
    prompt = torch.from_numpy(g["prompt"]).to(DEV)
    gen = gen if gen is not None else g["tokens_bf16"].shape[1] - prompt.shape[1] - 1
    dec = BlockDiffusionDecoder(model, prompt.shape[0], prompt.shape[1], gen, mask_id=mask_id, stop_id=stop_id,
                                pad_id=pad_id, schedule="static", **kw)
    return g, model, dec, prompt


@KV_STORE
def test_teacher_forced_static_schedule_matches_reference(fused):
    g, m, dec, prompt = _setup(fused_kv_store=fused)
    st = dec.st
    st.lens.zero_()
    n_gated = n_ok = n_all = n_all_ok = 0
    worst = []
    kinds = []
    with torch.no_grad():
        for i in range(int(g["n_trace"])):
            kind = int(g[f"t{i}_kind"])
            kinds.append(kind)
            ids = torch.from_numpy(g[f"t{i}_ids"]).to(DEV)
            T = ids.shape[1]
            pos = st.lens.to(torch.long)[:, None] + torch.arange(T, device=DEV)[None, :]
            if kind == 0:
                h = st.forward_commit(ids, pos, all_rows=True, mask_block=0)
            else:
                assert kind == 3
                lens0 = st.lens.clone()
                h = m.rmsnorm(st.forward_scratch(ids, pos), m.norm)
                assert torch.equal(st.lens, lens0), "a diffusion step must not move the committed length"
            logits = m.logits_rows(h)
            got = torch.softmax(logits, dim=-1).argmax(-1).cpu().numpy()
            top = logits.float().max(-1).values.cpu().numpy()
            ref, gap = g[f"t{i}_argmax"], g[f"t{i}_gap"]
            gate = gap > NEAR_TIE_ULPS * _bf16_ulp(top)
            n_all += got.size
            n_all_ok += int((got == ref).sum())
            n_gated += int(gate.sum())
            n_ok += int(((got == ref) & gate).sum())
            for b, t in zip(*np.nonzero((got != ref) & gate)):
                worst.append((i, kind, int(b), int(t), float(gap[b, t])))
    assert _lib.last_device_error()[0] == 0
    assert kinds.count(0) >= 2 and kinds.count(3) > kinds.count(0)
    frac = n_ok / max(1, n_gated)
    floor = float(g["ref_tf_f32_agree_gated"])
    print(f"static schedule teacher-forced argmax agreement: {n_ok}/{n_gated} gated ({frac:.4f}), "
          f"{n_all_ok}/{n_all} all ({n_all_ok / n_all:.4f}); reference fp32-vs-bf16 floor {floor:.4f} gated")
    assert frac >= floor - 0.005, f"argmax mismatches outside near ties (trace, kind, b, pos, gap): {worst[:10]}"


def test_static_prefill_is_bidirectional_over_the_prompt():
    """The static sampler's prefill attends with no mask, so the rows of the
    prompt's first block see the second block's keys.  Layer 1's K/V of the
    first block depend on layer 0's attention output, so they differ between
    the unmasked prefill and the dKV sampler's block-causal one."""
    g, m, dec, prompt = _setup(gen=64)
    assert prompt.shape[1] >= 64
    pos = torch.arange(prompt.shape[1], device=DEV).unsqueeze(0).expand(prompt.shape[0], -1)
    with torch.no_grad():
        dec.st.lens.zero_()
        dec.st.forward_commit(prompt, pos, mask_block=0)
        k_full = dec.st.k[1][:, :32].clone()
        dec.st.lens.zero_()
        dec.st.forward_commit(prompt, pos)
        k_blk = dec.st.k[1][:, :32].clone()
    assert not torch.equal(k_full, k_blk)


@KV_STORE
def test_free_running_static_decode_reported(fused):
    g, m, dec, prompt = _setup(fused_kv_store=fused)
    with torch.no_grad():
        out, _ = dec.generate(prompt)
    ref = g["tokens_bf16"]
    P = prompt.shape[1]
    got = out.cpu().numpy()
    assert got.shape == ref.shape
    assert np.array_equal(got[:, :P], ref[:, :P])
    agree = float((got[:, P:] == ref[:, P:]).mean())
    print(f"static schedule free-running agreement vs reference bf16: {agree:.4f} "
          f"(reference bf16-vs-fp32: {float(g['ref_bf16_vs_f32_gen_agreement']):.4f})")
    assert int((got[:, P:] == int(g["ids_special"][0])).sum()) == 0, "masks left in the output"
    assert _lib.last_device_error()[0] == 0


def test_static_graph_replay_identical_to_eager():
    g, m, dec, prompt = _setup(gen=64)
    with torch.no_grad():
        eager, _ = dec.generate(prompt, n_blocks=2)
        _, _, dec_g, _ = _setup(gen=64, use_graphs=True)
        dec_g.m = m
        dec_g.st.model = m
        dec_g.capture_all()
        assert set(dec_g._graphs) == {"begin", "full", "commit"}
        graphed, _ = dec_g.generate(prompt, n_blocks=2)
    assert torch.equal(eager, graphed)
