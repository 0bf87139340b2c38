"""Golden logits of ONE full dKV diffusion step of the REFERENCE model
(``Fast_dLLM_QwenForCausalLM.forward_dkv(is_full_step=True)``,
modeling.py:1625-1662) after a prompt prefill (``forward`` with
``update_past_key_values=True``), on the seeded tiny model of
make_golden_decode.py, run on CPU in bf16 and in fp32.

Usage:  python tests/golden/make_golden_dkv_step.py [/path/to/reference]

The fixture holds the prompt, the block tokens, the prefix K/V the prefill
left in the reference's cache (per layer, BHSD) and the step's logits.  It
pins ``oracle/torch_port.dkv_full_step_forward`` -- the CPU baseline and the
reference arm of bench.py -- to the reference's own forward.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import make_golden_decode as G  # noqa: E402  (shims, tiny geometry, weight construction)

PROMPT_LEN = 48  # not a multiple of the 32-token block: the block straddles a mask-grid boundary
BLOCK = 32


def run(dtype):
    modeling, _, cfg_cls = G.load_reference()
    model = G.build_reference_model(modeling, cfg_cls, dtype)
    g = torch.Generator().manual_seed(G.SEED + 7)
    prompt = torch.randint(0, 1000, (G.B, PROMPT_LEN), generator=g)
    block = torch.randint(0, 1000, (G.B, BLOCK), generator=g)
    block[:, 1:] = G.MASK_ID
    block[1, 5] = 17
    with torch.no_grad():
        out = model.forward(input_ids=prompt, use_cache=True, past_key_values=None, update_past_key_values=True,
                            block_size=BLOCK)
        pkv = out.past_key_values
        pk = [pkv.layers[l].keys.clone() for l in range(G.GEO["layers"])]
        pv = [pkv.layers[l].values.clone() for l in range(G.GEO["layers"])]
        step = model.forward_dkv(input_ids=block, use_cache=True, past_key_values=pkv, dkv_store=None,
                                 fed_indices=None, is_full_step=True)
    return prompt, block, pk, pv, step.logits


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    rec = {}
    for name, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
        prompt, block, pk, pv, logits = run(dt)
        rec[f"logits_{name}"] = logits.float().numpy()
        for l in range(len(pk)):
            rec[f"pk{l}_{name}"] = pk[l].float().numpy()
            rec[f"pv{l}_{name}"] = pv[l].float().numpy()
    np.savez_compressed(HERE / "dkv_step.npz", prompt=prompt.numpy(), block=block.numpy(),
                        seed=np.int64(G.SEED), init_std=np.float64(G.INIT_STD),
                        geo=np.array([G.GEO[k] for k in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn",
                                                         "vocab")]), **rec)
    print("logits", rec["logits_bf16"].shape, "prefix", rec["pk0_bf16"].shape)


if __name__ == "__main__":
    main()
