"""Pins the numpy restatements of the decode-forward stages next to the KV
path against the reference's own torch formulas run on the CPU in bf16
(oracle/torch_port.py: apply_rotary_pos_emb, Fast_dLLM_QwenRMSNorm; the MLP's
act_fn(gate) * up; the decoder layer's residual add)."""
import numpy as np
import torch
import torch.nn.functional as F

from oracle import kvcache_oracle as O
from oracle import torch_port


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def rbf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def test_swiglu_oracle_matches_torch_bf16():
    gu = rbf16((64, 2 * 512), 1, 3.0)
    ref = F.silu(gu[:, :512]) * gu[:, 512:]
    got = O.swiglu(bits(gu))
    # cos/exp of numpy vs torch's CPU kernels may differ in the last fp32 bit
    assert np.mean(got != bits(ref)) < 2e-3


def test_rope_oracle_matches_reference_rotary_embedding():
    rows, hq, hkv, D = 40, 4, 2, 128
    y = rbf16((rows, (hq + 2 * hkv) * D), 2)
    pos = np.arange(1000, 1000 + rows)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
    q, k, v = O.rope_qkv(bits(y), pos, inv.numpy(), hq, hkv)
    # the reference: fp32 angles, cos/sin rounded to the hidden dtype, bf16 ops
    f = torch.from_numpy(pos).float()[:, None] * inv[None, :]
    emb = torch.cat((f, f), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16)[None], emb.sin().to(torch.bfloat16)[None]
    x = y.view(1, rows, hq + 2 * hkv, D).transpose(1, 2)  # BHSD
    ref = torch_port.rope(x[:, : hq + hkv], cos, sin).transpose(1, 2)[0]
    assert np.mean(np.concatenate([q, k], axis=1) != bits(ref)) < 2e-3
    assert np.array_equal(v, bits(y.view(rows, hq + 2 * hkv, D)[:, hq + hkv:]))


def test_add_rmsnorm_oracle_matches_residual_then_reference_norm():
    x, res = rbf16((33, 3584), 3), rbf16((33, 3584), 4)
    w = (1 + 0.1 * torch.randn(3584, generator=torch.Generator().manual_seed(5))).to(torch.bfloat16)
    s_bits, n_bits = O.add_rmsnorm_bf16(bits(x), bits(res), bits(w), 1e-6)
    h = x + res  # the decoder layer's residual add, bf16
    assert np.array_equal(s_bits, bits(h))
    ref = torch_port.rmsnorm(h, w, 1e-6)
    d = np.abs(O.bf16_to_f32(n_bits) - ref.float().numpy())
    assert (d <= 2e-2 + 1e-2 * np.abs(ref.float().numpy())).all()
    assert np.mean(n_bits != bits(ref)) < 0.01
