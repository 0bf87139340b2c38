"""The reference's compiled execution mode on the drop-in classes:
FAST_DLLM_EXECUTION_MODE=compile swaps every attention layer to a branch-free
forward (patch_attention_layers_compiled, utils/attention_backends.py:901-974)
and compiles the diffusion step (utils/dynamo_utils.py:218-288).  Here a tiny
attention stack on StaticKVCache runs one block the way the static sampler
(generation_functions.py:243) drives it: a committed prefix through the eager
patched forward, then diffusion steps that write the block at kv_write_start
(prepare_write_idx -> write_scratch_compiled) and attend over scratch_seqlens
-- traced with torch.compile(fullgraph=True), so any graph break in the fdl
ops fails the test -- and finally the block's commit.  Outputs and scratch
K/V match the eager step (bit for bit without inductor's own fusions, within
the bf16 tolerance with them) and the CPU oracle's attention."""
import pytest
import torch

from fast_v2_b200 import _lib
from fast_v2_b200.utils import (StaticKVCache, get_attention_backend, patch_attention_layers,
                                patch_attention_layers_compiled, unpatch_attention_layers)
from oracle import kvcache_oracle as O
from tests._util import assert_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
ATOL, RTOL = 2e-2, 1e-2
L, B, HIDDEN, HQ, HKV, D, S, P, BLK = 2, 2, 256, 4, 2, 128, 256, 64, 32


@pytest.fixture(autouse=True)
def _clean():
    _lib.ensure_ops()
    _lib.last_device_error()
    yield
    assert _lib.last_device_error()[0] == 0


class _Attn(torch.nn.Module):
    def __init__(self, layer_idx):
        super().__init__()
        self.layer_idx, self.head_dim, self.scaling = layer_idx, D, D ** -0.5
        self.q_proj = torch.nn.Linear(HIDDEN, HQ * D)
        self.k_proj = torch.nn.Linear(HIDDEN, HKV * D)
        self.v_proj = torch.nn.Linear(HIDDEN, HKV * D)
        self.o_proj = torch.nn.Linear(HQ * D, HIDDEN, bias=False)

    def forward(self, *a, **k):  # replaced by the patch
        raise AssertionError("unpatched forward called")


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList()
        for i in range(L):
            layer = torch.nn.Module()
            layer.self_attn = _Attn(i)
            self.model.layers.append(layer)


def _rope(n, start):
    pos = torch.arange(start, start + n, device=DEV, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=DEV).float() / D))
    f = pos[:, None] * inv[None, :]
    emb = torch.cat((f, f), -1)
    return (emb.cos().to(torch.bfloat16)[None].expand(B, -1, -1).contiguous(),
            emb.sin().to(torch.bfloat16)[None].expand(B, -1, -1).contiguous())


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_scratch_steps_of_a_block_match_eager_and_oracle(backend):
    torch.manual_seed(0)
    torch._dynamo.reset()
    m = _Model().to(DEV).to(torch.bfloat16).requires_grad_(False)
    be = get_attention_backend()
    cache = StaticKVCache(B, S, L, HKV, D, torch.bfloat16, DEV)

    # committed prefix: the eager patched forward with update_past_key_values
    orig = patch_attention_layers(m, be)
    xp = torch.randn(B, P, HIDDEN, device=DEV).to(torch.bfloat16)
    cs = _rope(P, 0)
    with torch.no_grad():
        for l in range(L):
            m.model.layers[l].self_attn.forward(xp, cs, past_key_value=cache, update_past_key_values=True)
    unpatch_attention_layers(m, orig)
    assert cache.get_seq_length() == P

    # diffusion steps of the next block on the compiled, branch-free forward
    orig = patch_attention_layers_compiled(m, be)
    cache.set_kv_write_start(P)
    cache.prepare_write_idx(BLK)
    cache.set_scratch_seqlens(P + BLK)
    cos, sin = _rope(BLK, P)

    def step(x, cos, sin):
        return [m.model.layers[l].self_attn.forward(x, (cos, sin), past_key_value=cache) for l in range(L)]

    compiled = torch.compile(step, fullgraph=True, backend=backend)
    exact = backend == "aot_eager"
    for it in range(3):
        x = torch.randn(B, BLK, HIDDEN, device=DEV).to(torch.bfloat16)
        with torch.no_grad():
            eager = step(x, cos, sin)
            k_e = [cache.key_cache[l][:, P:P + BLK].clone() for l in range(L)]
            v_e = [cache.value_cache[l][:, P:P + BLK].clone() for l in range(L)]
            for l in range(L):  # the compiled step must write the scratch rows itself
                cache.key_cache[l][:, P:P + BLK].zero_()
                cache.value_cache[l][:, P:P + BLK].zero_()
            got = compiled(x, cos, sin)
        torch.cuda.synchronize()
        for l in range(L):
            kc, vc = cache.key_cache[l][:, P:P + BLK], cache.value_cache[l][:, P:P + BLK]
            if exact:
                assert torch.equal(got[l], eager[l]) and torch.equal(kc, k_e[l]) and torch.equal(vc, v_e[l])
            else:
                assert_close(f"step {it} K layer {l}", kc.float().cpu().numpy(), k_e[l].float().cpu().numpy(), ATOL,
                             RTOL)
                assert_close(f"step {it} out layer {l}", got[l].float().cpu().numpy(),
                             eager[l].float().cpu().numpy(), ATOL, RTOL)
            # the attention itself against the oracle over prefix + scratch block
            a = m.model.layers[l].self_attn
            q = a.q_proj(x).view(B, BLK, HQ, D)
            qe = q * cos.unsqueeze(2) + torch.cat((-q[..., D // 2:], q[..., :D // 2]), -1) * sin.unsqueeze(2)
            ref = O.block_attention(qe.float().cpu().numpy(), cache.key_cache[l].float().cpu().numpy(),
                                    cache.value_cache[l].float().cpu().numpy(), [P + BLK] * B)
            ctx = torch.from_numpy(ref).to(DEV).to(torch.bfloat16).reshape(B, BLK, -1)
            assert_close(f"step {it} oracle layer {l}", got[l].float().cpu().numpy(),
                         a.o_proj(ctx).float().cpu().numpy(), 5e-2, 5e-2)
    # the committed length did not move during the scratch steps
    assert cache.get_seq_length() == P
    unpatch_attention_layers(m, orig)

    # commit of the decoded block: the eager patched forward appends it
    orig = patch_attention_layers(m, be)
    with torch.no_grad():
        for l in range(L):
            m.model.layers[l].self_attn.forward(x, (cos, sin), past_key_value=cache, update_past_key_values=True)
    unpatch_attention_layers(m, orig)
    assert cache.get_seq_length() == P + BLK
