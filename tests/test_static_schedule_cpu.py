"""CPU checks of the static-cache schedule: the golden trace of the
reference's batch_sample_dynamo (tests/golden/decode_static.npz) has the
shape that sampler produces, and the decoder refuses schedule combinations
the reference does not have."""
import numpy as np
import pytest

from fast_v2_b200.block_decode import BlockDiffusionDecoder
from tests._util import golden


def test_static_trace_structure():
    g = golden("decode_static")
    n = int(g["n_trace"])
    kinds = [int(g[f"t{i}_kind"]) for i in range(n)]
    P = g["prompt"].shape[1]
    B = g["prompt"].shape[0]
    gen = g["tokens_bf16"].shape[1] - P - 1
    # prefill, then per block: diffusion steps (kind 3), then one commit (kind 0)
    assert kinds[0] == 0 and g["t0_ids"].shape == (B, P)
    assert set(kinds) == {0, 3}
    assert kinds.count(0) == 1 + gen // 32
    assert kinds[-1] == 0
    for i in range(1, n):
        ids = g[f"t{i}_ids"]
        assert ids.shape == (B, 32)
        assert g[f"t{i}_argmax"].shape == (B, 32) and g[f"t{i}_gap"].shape == (B, 32)
        if kinds[i] == 3 and kinds[i - 1] == 0:
            # a block starts as [bridge token, 31 masks]
            assert (ids[:, 1:] == int(g["ids_special"][0])).all()
    # every block takes at least 4 steps (one per 8-token sub-block)
    starts = [i for i in range(1, n) if kinds[i] == 3 and kinds[i - 1] == 0]
    ends = [i for i in range(1, n) if kinds[i] == 0]
    assert all(e - s >= 4 for s, e in zip(starts, ends))
    # the reference's own fp32 path agrees with its bf16 path outside near ties
    assert float(g["ref_tf_f32_agree_gated"]) > 0.99


def test_static_schedule_argument_checks():
    with pytest.raises(ValueError):
        BlockDiffusionDecoder(None, 2, 64, 64, schedule="dynamo")
    with pytest.raises(ValueError):
        BlockDiffusionDecoder(None, 2, 64, 64, schedule="static", sparse_keep=0.25)


def test_static_trace_prompt_matches_dkv_trace_prompt():
    """Both golden decodes start from the same seeded prompt and weights."""
    a, b = golden("decode_static"), golden("decode_dkv")
    assert np.array_equal(a["prompt"], b["prompt"])
    assert int(a["seed"]) == int(b["seed"]) and np.array_equal(a["geo"], b["geo"])
