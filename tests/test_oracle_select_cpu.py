"""Pin the selection oracle (oracle/select_oracle.py) to the reference's own
functions -- _focus_importance, _focus_select and the cosine top-k of the
sparse forward -- through golden vectors (tests/golden/make_golden.py,
select.npz), and restate the reference's known-answer tests for them
(tests/test_focus.py:32-124 of the reference).  CPU only."""
import numpy as np

from oracle import kvcache_oracle as O
from oracle import select_oracle as SO
from tests._util import assert_close, golden


def _f(g, key, tag):
    a = g[key]
    return O.bf16_to_f32(a) if tag == "bf16" else a.astype(np.float32)


def test_focus_importance_matches_reference():
    g = golden("select")
    for tag in ("bf16", "f32"):
        q, k = _f(g, f"imp_{tag}_q", tag), _f(g, f"imp_{tag}_k", tag)
        got = SO.focus_importance(q, k, g[f"imp_{tag}_mask"], q.shape[-1] ** -0.5, tag == "bf16")
        assert_close(f"importance {tag}", got, g[f"imp_{tag}_out"], 2e-2, 1e-2)
        assert np.all(got[1] == 0)  # nothing masked in row 1: no importance


def test_focus_select_matches_reference_exactly():
    g = golden("select")
    for tag in ("bf16", "f32"):
        for i in range(int(g[f"sel_{tag}_n"])):
            key = f"sel_{tag}_{i}"
            avg, alpha, ro = g[f"{key}_args"]
            S = g[f"{key}_mask"].shape[1]
            K = SO.focus_retain_k(S, avg, alpha, None if np.isnan(ro) else ro)
            frozen = g[f"{key}_frozen"] if bool(g[f"{key}_has_frozen"]) else None
            idx, ksel = SO.focus_select(_f(g, f"{key}_delta", tag), g[f"{key}_mask"], K, tag == "bf16", frozen)
            assert ksel == int(g[f"{key}_ksel"]), (tag, i)
            assert np.array_equal(idx, g[f"{key}_idx"][:, :ksel]), (tag, i)


def test_cosine_select_matches_reference():
    g = golden("select")
    for tag in ("bf16", "f32"):
        h, c = _f(g, f"cos_{tag}_hidden", tag), _f(g, f"cos_{tag}_cached", tag)
        idx, cos = SO.cosine_select(h, c, int(g[f"cos_{tag}_n"]), tag == "bf16")
        if tag == "bf16":
            # every rounding point of torch's bf16 cosine_similarity reproduced
            assert np.array_equal(cos, g[f"cos_{tag}_cos"])
        else:
            assert_close("cos f32", cos, g[f"cos_{tag}_cos"], 1e-6, 1e-6)
        assert np.array_equal(idx, g[f"cos_{tag}_idx"])


# ---- the reference's known-answer tests (tests/test_focus.py:32-124), fp32 ----


def test_known_answer_importance_shape_and_masking():
    rng = np.random.default_rng(0)
    B, H, S, d = 2, 4, 6, 8
    q = rng.standard_normal((B, H, S, d)).astype(np.float32)
    k = rng.standard_normal((B, H, S, d)).astype(np.float32)
    mask = np.zeros((B, S), bool)
    mask[:, 2:] = True
    imp = SO.focus_importance(q, k, mask, d ** -0.5, False)
    assert imp.shape == (B, S)
    assert np.allclose(imp[:, :2], 0.0, atol=1e-5)
    assert np.all(imp[:, 2:] > 0)


def test_known_answer_select_respects_rule_and_budget():
    delta = np.array([[-9., -9., 0.1, 0.2, 5.0, 4.0]], np.float32)
    mask = np.array([[False, False, True, True, True, True]])
    idx, ksel = SO.focus_select(delta, mask, SO.focus_retain_k(6, 2.0, 1.0), False)
    assert idx.shape[1] == ksel
    sel = set(idx[0].tolist())
    assert {0, 1, 4, 5}.issubset(sel) and 2 not in sel


def test_known_answer_select_always_retains_decoded():
    delta = np.zeros((1, 8), np.float32)
    delta[0, 7] = 5.0
    mask = np.array([[False, False, False, True, True, True, True, True]])
    idx, _ = SO.focus_select(delta, mask, SO.focus_retain_k(8, 1.0, 1.0), False)
    sel = set(idx[0].tolist())
    assert {0, 1, 2}.issubset(sel) and 7 in sel


def test_known_answer_select_retain_all_override():
    delta = np.random.default_rng(1).standard_normal((1, 8)).astype(np.float32)
    mask = np.ones((1, 8), bool)
    idx, ksel = SO.focus_select(delta, mask, SO.focus_retain_k(8, 1.0, 1.0, 1.0), False)
    assert ksel == 8 and idx[0].tolist() == list(range(8))


def test_equal_values_rank_by_position():
    """torch.topk leaves equal values unordered; the fixed rule here (and in
    the kernels) is lower index first, for largest and smallest."""
    v = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]])
    assert SO.rank_select(v, 2, largest=True)[0].tolist() == [False, True, True, False, False]
    assert SO.rank_select(v, 3, largest=False)[0].tolist() == [True, True, False, True, False]
    assert SO.butterfly_sum(np.arange(32, dtype=np.float32)[None])[0] == 496.0


def test_focus_select_invariants_on_random_blocks():
    """Properties _focus_select guarantees (modeling.py:240-306): every
    decoded, non-frozen token is kept; Ksel >= the retain target (unless
    frozen tokens cap it); indices ascend without repeats; frozen tokens only
    appear as padding once every non-frozen token is in."""
    rng = np.random.default_rng(12)
    for trial in range(300):
        B, S = 3, 32
        bf = trial % 2 == 0
        d = SO.rnd(rng.standard_normal((B, S)).astype(np.float32) * 0.5, bf)
        mask = rng.random((B, S)) < rng.random()
        frozen = (rng.random((B, S)) < 0.3) & ~mask if trial % 3 == 0 else None
        K = SO.focus_retain_k(S, 1.0 + trial % 6, 1.5)
        idx, ksel = SO.focus_select(d, mask, K, bf, frozen)
        assert idx.shape == (B, ksel) and 1 <= ksel <= S
        if frozen is None:
            assert ksel >= K
        for b in range(B):
            row = idx[b].tolist()
            assert row == sorted(set(row))
            fz = frozen[b] if frozen is not None else np.zeros(S, bool)
            keep = set(np.nonzero(~mask[b] & ~fz)[0].tolist())
            assert keep.issubset(row), (trial, b)
            if any(fz[i] for i in row):
                assert set(np.nonzero(~fz)[0].tolist()).issubset(row), (trial, b)


def test_cosine_select_invariants():
    """The selection holds the n lowest similarities (ties by position) and
    a token identical to its cached input is never chosen before a changed one."""
    rng = np.random.default_rng(13)
    for trial in range(20):
        B, S, H = 2, 32, 256
        bf = trial % 2 == 0
        h = SO.rnd(rng.standard_normal((B, S, H)).astype(np.float32), bf)
        c = h.copy()
        moved = rng.random((B, S)) < 0.3
        c[moved] = SO.rnd(rng.standard_normal((int(moved.sum()), H)).astype(np.float32), bf)
        n = int(rng.integers(1, S))
        idx, cos = SO.cosine_select(h, c, n, bf)
        for b in range(B):
            sel = set(idx[b].tolist())
            worst = max(cos[b, list(sel)])
            assert all(cos[b, i] >= worst for i in range(S) if i not in sel)
            if n <= int(moved[b].sum()):
                assert sel.issubset(set(np.nonzero(moved[b])[0].tolist())), (trial, b)
