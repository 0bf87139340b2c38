"""The greedy-sampling oracle (softmax -> argmax -> gathered probability, bf16)
pinned to the torch ops the reference's sampler calls
(sample_with_top_p at temperature 0, modeling.py:2263-2269, and the x1_p gather
of generation_functions.py:2290-2291), run here on the CPU."""
import numpy as np
import pytest
import torch

from oracle import kvcache_oracle as O
from tests._util import bits_of


def _reference(logits_bf16):
    p = torch.softmax(logits_bf16, dim=-1)
    x1 = p.argmax(dim=-1)
    return x1.numpy(), bits_of(torch.gather(p, -1, x1[:, None])[:, 0])


@pytest.mark.parametrize("rows,vocab,scale,seed", [(64, 1000, 3.0, 0), (32, 4099, 1.0, 1), (48, 777, 0.05, 2),
                                                    (16, 152064, 2.0, 3)])
def test_oracle_matches_torch_softmax_argmax(rows, vocab, scale, seed):
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(rows, vocab, generator=g) * scale).to(torch.bfloat16)
    tok, prob = O.softmax_argmax_bf16(bits_of(logits))
    rt, rp = _reference(logits)
    assert np.array_equal(tok, rt)
    # the probability may differ by one bf16 ulp when 1/s sits on a rounding boundary
    assert np.abs(prob.astype(np.int32) - rp.astype(np.int32)).max() <= 1


def test_ties_go_to_the_first_index():
    # Small logits: many entries share the largest bf16 probability.
    logits = torch.zeros(4, 300, dtype=torch.bfloat16)
    logits[0, 7] = logits[0, 3] = 1.0
    logits[1, 299] = 0.5
    logits[2, 10:20] = 0.25
    tok, _ = O.softmax_argmax_bf16(bits_of(logits))
    assert tok.tolist() == [3, 299, 10, 0]
    assert np.array_equal(tok, _reference(logits)[0])
