"""oracle/torch_port.dkv_full_step_forward -- the reference arm and CPU
baseline of bench.py, and the fp32 reference of the config-4/5 agreement test --
pinned to the reference's own full dKV step (forward_dkv with
is_full_step=True, modeling.py:1625-1662) after a prefill, recorded by
tests/golden/make_golden_dkv_step.py on the seeded tiny model, in fp32 and
bf16: the port performs the same torch operations in the same order, so its
logits are identical bit for bit."""
import numpy as np
import pytest
import torch

from fast_v2_b200.block_decode import BlockDiffusionLM, Geometry
from oracle import torch_port
from tests._util import golden


def _port_layers(model, geo):
    hq, hk = geo.heads * geo.head_dim, geo.kv_heads * geo.head_dim
    out = []
    for w in model.layers:
        out.append(dict(wq=w["wqkv"][:hq], bq=w["bqkv"][:hq], wk=w["wqkv"][hq:hq + hk], bk=w["bqkv"][hq:hq + hk],
                        wv=w["wqkv"][hq + hk:], bv=w["bqkv"][hq + hk:], wo=w["wo"], ln1=w["ln1"], ln2=w["ln2"],
                        wg=w["wgu"][:geo.ffn], wu=w["wgu"][geo.ffn:], wd=w["wd"]))
    return out


@pytest.mark.parametrize("name,dtype", [("f32", torch.float32), ("bf16", torch.bfloat16)])
def test_port_full_dkv_step_matches_reference_forward_dkv(name, dtype):
    g = golden("dkv_step")
    L, H, hq, hkv, d, ffn, V = (int(x) for x in g["geo"])
    geo = Geometry(L, H, hq, hkv, d, ffn, V)
    model = BlockDiffusionLM(geo, device="cpu", dtype=dtype, seed=int(g["seed"]), init_std=float(g["init_std"]),
                             init_device="cpu", load_ops=False)
    geod = dict(head_dim=d, heads=hq, kv_heads=hkv, rope_theta=geo.rope_theta, eps=geo.eps, layers=L, hidden=H)
    pk = [torch.from_numpy(g[f"pk{l}_{name}"]).to(dtype) for l in range(L)]
    pv = [torch.from_numpy(g[f"pv{l}_{name}"]).to(dtype) for l in range(L)]
    ids = torch.from_numpy(g["block"])
    past = int(g["prompt"].shape[1])
    with torch.no_grad():
        got = torch_port.dkv_full_step_forward(_port_layers(model, geo), model.embed, model.norm, model.lm_head, ids,
                                               pk, pv, past, geod).float().numpy()
    ref = g[f"logits_{name}"]
    assert got.shape == ref.shape
    diff = np.abs(got - ref)
    print(f"{name}: max |port - reference| = {diff.max():.3e} (logit scale {np.abs(ref).max():.3f}); "
          f"argmax agreement {(got.argmax(-1) == ref.argmax(-1)).mean():.4f}")
    assert np.array_equal(got, ref)
