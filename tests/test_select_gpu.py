"""Token selection kernels (fdl_cosine_select, fdl_focus_select,
fdl_focus_importance) against the reference's own outputs (golden vectors
from tests/golden/make_golden.py) and the CPU oracle (oracle/select_oracle.py):
bit-exact indices and widths, importance within bf16 tolerance."""
import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib, focus
from oracle import kvcache_oracle as O
from oracle import select_oracle as SO
from tests._util import assert_close, golden, t_from_bits

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(autouse=True)
def _clean():
    _lib.ensure_ops()
    _lib.last_device_error()
    yield
    assert _lib.last_device_error()[0] == 0


def _dev(g, key, tag):
    a = g[key]
    return t_from_bits(a, DEV) if tag == "bf16" else torch.from_numpy(a).to(DEV)


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("tag", ["bf16", "f32"])
def test_cosine_select_matches_reference_and_refreshes_cache(tag):
    g = golden("select")
    h, c = _dev(g, f"cos_{tag}_hidden", tag), _dev(g, f"cos_{tag}_cached", tag)
    B, S, _ = h.shape
    cos = torch.empty(B, S, dtype=torch.float32, device=DEV)
    idx = focus.cosine_select(h, c, int(g[f"cos_{tag}_n"]), refresh_cache=True, cos_out=cos)
    assert np.array_equal(idx.cpu().numpy(), g[f"cos_{tag}_idx"])
    _, ocos = SO.cosine_select(_np(h), _np(_dev(g, f"cos_{tag}_cached", tag)), int(g[f"cos_{tag}_n"]), tag == "bf16")
    assert np.array_equal(cos.cpu().numpy(), ocos)  # same reduction order as the oracle: bit for bit
    if tag == "bf16":
        assert np.array_equal(cos.cpu().numpy(), g[f"cos_{tag}_cos"])  # and as torch's bf16 op
    assert torch.equal(c, h)  # cache refreshed with the new layer input


def test_cosine_select_at_decode_size_equals_oracle():
    """64 sequences x 32 tokens of the 7B hidden size, bf16, with ties in the
    bf16 similarities (lower index wins)."""
    gen = torch.Generator().manual_seed(21)
    B, S, H = 64, 32, 3584
    h = torch.randn(B, S, H, generator=gen)
    c = h + 0.05 * torch.randn(B, S, H, generator=gen) * torch.rand(B, S, 1, generator=gen)
    hb, cb = h.to(torch.bfloat16), c.to(torch.bfloat16)
    cos = torch.empty(B, S, dtype=torch.float32, device=DEV)
    idx = focus.cosine_select(hb.to(DEV), cb.to(DEV), 8, cos_out=cos)
    oidx, ocos = SO.cosine_select(hb.float().numpy(), cb.float().numpy(), 8, True)
    assert np.array_equal(cos.cpu().numpy(), ocos)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert len(np.unique(ocos)) < ocos.size  # the case does contain ties


@pytest.mark.parametrize("tag", ["bf16", "f32"])
def test_focus_select_matches_reference(tag):
    g = golden("select")
    for i in range(int(g[f"sel_{tag}_n"])):
        key = f"sel_{tag}_{i}"
        avg, alpha, ro = g[f"{key}_args"]
        frozen = torch.from_numpy(g[f"{key}_frozen"]).to(DEV) if bool(g[f"{key}_has_frozen"]) else None
        idx, ksel = focus.focus_select(_dev(g, f"{key}_delta", tag), torch.from_numpy(g[f"{key}_mask"]).to(DEV),
                                       float(avg), float(alpha), None if np.isnan(ro) else float(ro), frozen=frozen)
        assert ksel == int(g[f"{key}_ksel"]), (tag, i)
        assert np.array_equal(idx.cpu().numpy(), g[f"{key}_idx"][:, :ksel]), (tag, i)


def test_focus_select_ties_and_frozen_padding_equal_oracle():
    """Many equal deltas and rows padded with frozen positions: the cases
    where torch.topk's order is open; kernel and oracle both rank equal
    values by position."""
    rng = np.random.default_rng(4)
    for trial in range(60):
        B, S = 5, 32
        bf = trial % 2 == 0
        d = (rng.integers(-4, 5, size=(B, S)) * 0.25).astype(np.float32)
        mask = rng.random((B, S)) < 0.2 + 0.6 * (trial % 5) / 4
        frozen = (rng.random((B, S)) < 0.4) & ~mask if trial % 3 else None
        K = 1 + trial % 9
        dt = torch.bfloat16 if bf else torch.float32
        sel = torch.empty(B, S, dtype=torch.long, device=DEV)
        ks = torch.empty(1, dtype=torch.int32, device=DEV)
        torch.ops.fdl.focus_select(torch.from_numpy(d).to(dt).to(DEV), torch.from_numpy(mask).to(DEV),
                                   None if frozen is None else torch.from_numpy(frozen).to(DEV), K, sel, ks)
        oidx, oks = SO.focus_select(d, mask, K, bf, frozen)
        got = sel.cpu().numpy()
        assert int(ks.item()) == oks, trial
        assert np.array_equal(got[:, :oks], oidx), trial
        assert np.all(got[:, oks:] == -1), trial


@pytest.mark.parametrize("tag", ["bf16", "f32"])
def test_focus_importance_matches_reference(tag):
    g = golden("select")
    q, k = _dev(g, f"imp_{tag}_q", tag), _dev(g, f"imp_{tag}_k", tag)
    mask = torch.from_numpy(g[f"imp_{tag}_mask"]).to(DEV)
    imp = focus.focus_importance(q, k, mask, q.shape[-1] ** -0.5)
    assert imp.dtype == q.dtype
    assert_close(f"importance {tag}", _np(imp), g[f"imp_{tag}_out"], 2e-2, 1e-2)
    assert float(imp[1].abs().max()) == 0.0  # nothing masked in row 1


def test_focus_importance_7b_heads_gqa_equals_expanded():
    """28 query heads over 4 KV heads: the in-kernel head mapping equals the
    reference's repeat_kv input, and both match the oracle."""
    gen = torch.Generator().manual_seed(9)
    B, Hkv, rep, S, D = 8, 4, 7, 32, 128
    q = (torch.randn(B, Hkv * rep, S, D, generator=gen) * 1.5).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=gen).to(torch.bfloat16)
    mask = torch.rand(B, S, generator=gen) < 0.5
    mask[0] = True
    kx = k[:, :, None].expand(B, Hkv, rep, S, D).reshape(B, Hkv * rep, S, D)
    a = focus.focus_importance(q.to(DEV), k.to(DEV), mask.to(DEV), D ** -0.5)
    b = focus.focus_importance(q.to(DEV), kx.to(DEV), mask.to(DEV), D ** -0.5)
    assert torch.equal(a, b)
    ref = SO.focus_importance(q.float().numpy(), k.float().numpy(), mask.numpy(), D ** -0.5, True)
    assert_close("importance 7B heads", _np(a), ref, 2e-2, 1e-2)


def test_known_answers_of_the_reference_on_the_gpu():
    """tests/test_focus.py:32-124 of the reference, through the kernels (fp32)."""
    torch.manual_seed(0)
    B, H, S, d = 2, 4, 6, 8
    q, k = torch.randn(B, H, S, d, device=DEV), torch.randn(B, H, S, d, device=DEV)
    mask = torch.zeros(B, S, dtype=torch.bool, device=DEV)
    mask[:, 2:] = True
    imp = focus.focus_importance(q, k, mask, d ** -0.5)
    assert imp.shape == (B, S)
    assert torch.allclose(imp[:, :2], torch.zeros(B, 2, device=DEV), atol=1e-5) and bool((imp[:, 2:] > 0).all())
    delta = torch.tensor([[-9., -9., 0.1, 0.2, 5.0, 4.0]], device=DEV)
    m = torch.tensor([[False, False, True, True, True, True]], device=DEV)
    idx, ksel = focus.focus_select(delta, m, 2.0, 1.0)
    assert idx.shape[1] == ksel and {0, 1, 4, 5}.issubset(set(idx[0].tolist())) and 2 not in idx[0].tolist()
    delta = torch.zeros(1, 8, device=DEV)
    delta[0, 7] = 5.0
    m = torch.tensor([[False, False, False, True, True, True, True, True]], device=DEV)
    idx, _ = focus.focus_select(delta, m, 1.0, 1.0)
    assert {0, 1, 2, 7}.issubset(set(idx[0].tolist()))
    idx, ksel = focus.focus_select(torch.randn(1, 8, device=DEV), torch.ones(1, 8, dtype=torch.bool, device=DEV),
                                   1.0, 1.0, retain_override=1.0)
    assert ksel == 8 and idx[0].tolist() == list(range(8))
