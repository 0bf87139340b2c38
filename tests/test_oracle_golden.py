"""Pin the CPU oracle to golden vectors produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

from oracle import kvcache_oracle as O
from tests._util import assert_close, golden


def test_bf16_roundtrip_exact():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    b = O.f32_to_bf16(x)
    assert np.array_equal(O.f32_to_bf16(O.bf16_to_f32(b)), b)
    # RNE against torch's conversion
    import torch

    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(b, ref)


def test_static_kv_cache_sequence_matches_reference():
    g = golden("static_kv")
    L = 2
    B, S, H, D = g["final_k0"].shape
    for l in range(L):
        kc = np.zeros((B, S, H, D), np.uint16)
        vc = np.zeros_like(kc)
        O.kv_update_uniform(kc, vc, g[f"pre_k{l}"], g[f"pre_v{l}"], 0)
        O.kv_update_uniform(kc, vc, g[f"commit_k{l}"], g[f"commit_v{l}"], 40)
        # scratch write at kv_write_start = committed length, per-sequence form
        start = np.full(B, int(g["seq_len_after_commit"]), np.int32)
        O.kv_append(kc, vc, g[f"scratch_k{l}"], g[f"scratch_v{l}"], start)
        O.scatter_rows(kc, g[f"sparse_k{l}"], g["sparse_pos"])
        O.scatter_rows(vc, g[f"sparse_v{l}"], g["sparse_pos"])
        assert np.array_equal(kc, g[f"final_k{l}"]), f"K layer {l}"
        assert np.array_equal(vc, g[f"final_v{l}"]), f"V layer {l}"
    assert int(g["seq_len_after_commit"]) == 72
    assert np.all(g["cache_seqlens"] == 72)


def test_dynamic_block_kv_and_block_sparse_match_reference():
    g = golden("dynamic_block")
    fed, n = O.dkv_fed_indices(g["prv"])
    assert n == int(g["n_fed"]) and np.array_equal(fed, g["fed"])
    for l in range(2):
        k = g[f"full_k{l}"].copy()
        v = g[f"full_v{l}"].copy()
        O.scatter_rows(k, g[f"sel_k{l}"], g["fed"], seq_axis=2)
        O.scatter_rows(v, g[f"sel_v{l}"], g["fed"], seq_axis=2)
        assert np.array_equal(k, g[f"final_k{l}"]) and np.array_equal(v, g[f"final_v{l}"])
    base = g["bsc_base"].copy()
    O.scatter_rows(base, g["bsc_vals"], g["bsc_tok"])
    assert np.array_equal(base, g["bsc_final"])


@pytest.mark.parametrize("tag", ["bf16", "f32"])
def test_gather_rmsnorm_matches_reference(tag):
    g = golden("rmsnorm")
    for i in range(int(g[f"{tag}_n"])):
        k = f"{tag}_{i}"
        if tag == "bf16":
            gath, normed = O.gather_rmsnorm_bf16(g[f"{k}_x"], g[f"{k}_idx"], g[f"{k}_w"], float(g[f"{k}_eps"]))
            assert np.array_equal(gath, g[f"{k}_gathered"])
            # fp32 reduction order differs (numpy float64 vs torch fp32): allow 1 bf16 ulp
            assert_close(k, O.bf16_to_f32(normed), O.bf16_to_f32(g[f"{k}_normed"]), atol=2e-2, rtol=1e-2)
            mism = np.mean(normed != g[f"{k}_normed"])
            assert mism < 0.01, f"{k}: {mism:.4f} of outputs differ in bits"
        else:
            gath, normed = O.gather_rmsnorm_f32(g[f"{k}_x"], g[f"{k}_idx"], g[f"{k}_w"], float(g[f"{k}_eps"]))
            assert np.array_equal(gath, g[f"{k}_gathered"])
            assert_close(k, normed, g[f"{k}_normed"], atol=1e-5, rtol=1e-5)


def test_attention_matches_reference_sdpa():
    g = golden("attention")
    q = O.bf16_to_f32(g["kv_q"])
    k = O.bf16_to_f32(g["kv_k"])
    v = O.bf16_to_f32(g["kv_v"])
    out = O.block_attention(q, k, v, g["kv_seqlens"])
    assert_close("static", out, g["kv_out"], atol=1e-4, rtol=1e-4)


def test_dynamic_attention_with_block_causal_mask_matches_reference():
    g = golden("attention")
    qd = O.bf16_to_f32(g["dyn_q"]).transpose(0, 2, 1, 3)  # BHSD -> BSHD
    pk = O.bf16_to_f32(g["dyn_pk"]).transpose(0, 2, 1, 3)
    pv = O.bf16_to_f32(g["dyn_pv"]).transpose(0, 2, 1, 3)
    bk = O.bf16_to_f32(g["dyn_bk"]).transpose(0, 2, 1, 3)
    bv = O.bf16_to_f32(g["dyn_bv"]).transpose(0, 2, 1, 3)
    P = pk.shape[1]
    out = O.block_attention(qd, pk, pv, np.array([P]), k_blk=bk, v_blk=bv, mask_block=32)
    assert_close("dynamic", out, g["dyn_out"], atol=1e-4, rtol=1e-4)
    # the mask the oracle applies is the reference's eval_mask
    assert np.array_equal(O.eval_block_mask(32, 32, P), g["dyn_mask"])
    # cat + repeat_kv
    cat = O.concat_bhsd(g["dyn_pk"], g["dyn_bk"])
    assert np.array_equal(np.repeat(cat, 7, axis=1), g["dyn_repeat_k"])


def test_index_ops_match_reference():
    g = golden("index_ops")
    for i in range(6):
        fed, n = O.dkv_fed_indices(g[f"fed_prv_{i}"])
        assert n == int(g[f"fed_n_{i}"]) and np.array_equal(fed, g[f"fed_idx_{i}"]), i
        assert np.array_equal(O.focus_update_frozen(g[f"frz_in_{i}"], g[f"frz_mask_{i}"]), g[f"frz_out_{i}"])
    for cl in (0, 40, 64):
        assert np.array_equal(O.eval_block_mask(32, 32, cl), g[f"eval_mask_{cl}"])


def test_sparse_prefix_spec_properties():
    """No reference counterpart: check the specification's own properties."""
    rng = np.random.default_rng(3)
    B, cap, H, D = 3, 300, 4, 128
    k = O.f32_to_bf16(rng.standard_normal((B, cap, H, D)).astype(np.float32))
    lens = np.array([300, 1, 77], np.int32)
    # force ties: duplicate rows of row 0 at 5 and 9 in batch 0
    k[0, 5] = k[0, 9] = k[0, 0]
    sel, keep = O.sparse_prefix_select(k, lens)
    assert list(keep) == [75, 1, 20]
    score = O.key_norm_scores(k, lens)
    for b in range(B):
        s = sel[b, : keep[b]]
        assert np.all(np.diff(s) > 0)
        assert np.all(sel[b, keep[b]:] == -1)
        thr = score[b, s].min()
        rest = np.setdiff1d(np.arange(lens[b]), s)
        assert np.all(score[b, rest] <= thr)
    # fp32 score close to a float64 norm
    ref = np.sqrt((O.bf16_to_f32(k).astype(np.float64) ** 2).sum(axis=(2, 3)))
    assert_close("score", score[0], ref[0], atol=1e-4, rtol=1e-5)


_COMPACT_KEYS = ["skv_k0", "skv_v0", "skv_k1", "skv_v1", "sbc_k0", "sbc_v1", "dbk_k1", "dbk_v2"]


def test_batch_compaction_matches_reference():
    """Two compactions (5 -> 3 -> 2 slots) of every cache class: the
    out-of-place restatement and the in-place order of the CUDA kernel both
    give the reference's buffers."""
    g = golden("compaction")
    for key in _COMPACT_KEYS + ["cache_seqlens", "scratch_seqlens"]:
        cur = g[f"init_{key}"]
        inplace = cur.copy()
        n = cur.shape[0]
        for i in range(2):
            act = g[f"active_{i}"]
            cur = O.batch_compact(cur, act)
            assert O.batch_compact_in_place(inplace[:n], act)
            n = act.shape[0]
            assert np.array_equal(cur, g[f"step{i}_{key}"]), (key, i)
            assert np.array_equal(inplace[:n], g[f"step{i}_{key}"]), (key, i)
    for name in ("layer_input", "attn_output", "mlp_input", "mlp_output"):
        cur = g[f"init_bsc_{name}"]
        for i in range(2):
            cur = O.batch_compact(cur, g[f"active_{i}"], batch_axis=1)
            assert np.array_equal(cur, g[f"step{i}_bsc_{name}"]), (name, i)
    assert int(g["step1_batch"]) == 2 and int(g["restored_batch"]) == 5 and bool(g["restored_all_zero"])


def test_in_place_compaction_order_property():
    """For every list with i <= active[i] < batch (ascending distinct slots,
    repeats, out-of-order lists such as [3, 1]) the sequential in-place order
    equals the gather; every other list is refused with the buffer intact."""
    rng = np.random.default_rng(5)
    for trial in range(400):
        B = int(rng.integers(1, 12))
        buf = rng.integers(0, 1 << 16, size=(B, 6), dtype=np.uint16)
        n = int(rng.integers(0, B + 1))
        act = np.array([rng.integers(i, B) for i in range(n)], np.int64)
        if trial % 4 == 0:
            act = np.sort(rng.choice(B, size=n, replace=False)).astype(np.int64)
        want = O.batch_compact(buf, act)
        got = buf.copy()
        assert O.batch_compact_in_place(got, act)
        assert np.array_equal(got[:n], want)
        assert np.array_equal(got[n:], buf[n:])  # rows past the kept ones are never written
    for bad in ([1, 0], [0, 0], [2, 5]):
        buf = np.arange(12, dtype=np.uint16).reshape(4, 3)
        keep = buf.copy()
        assert not O.batch_compact_in_place(buf, np.array(bad)) and np.array_equal(buf, keep)


def test_decoder_fed_indices_match_reference():
    """The decoder's device-side _dkv_fed_indices (plain torch ops, run here on
    CPU tensors) against the reference's outputs: same indices and width, and
    with a fixed width the same rows padded further with the first index."""
    import torch

    from fast_v2_b200.block_decode import dkv_fed_indices

    g = golden("index_ops")
    for i in range(6):
        prv = torch.from_numpy(g[f"fed_prv_{i}"])
        fed, n = dkv_fed_indices(prv)
        assert n == int(g[f"fed_n_{i}"]) and np.array_equal(fed.numpy(), g[f"fed_idx_{i}"]), i
        wide, w = dkv_fed_indices(prv, 32)
        assert w == 32 and np.array_equal(wide[:, :n].numpy(), g[f"fed_idx_{i}"]), i
        assert np.all(wide[:, n:].numpy() == g[f"fed_idx_{i}"][:, :1]), i
