"""GPU parity of the fused greedy-sampling kernel (fdl_softmax_argmax) against
the CPU oracle and against the torch path the sampler used before (bf16
softmax, argmax, gather): the token bit-exact, the probability within one
bf16 ulp (1/s on a rounding boundary), at the 7B vocabulary and on tie-heavy
rows."""
import numpy as np
import pytest
import torch

from fast_v2_b200 import _lib
from oracle import kvcache_oracle as O
from tests._util import bits_of

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _ops():
    _lib.ensure_ops()
    _lib.last_device_error()
    yield
    code, info = _lib.last_device_error()
    assert code == 0, f"device error {code} (info {info}) left by the test"


def _fused(logits):
    rows = logits.numel() // logits.shape[-1]
    tok = torch.empty(rows, dtype=torch.long, device=DEV)
    prob = torch.empty(rows, dtype=torch.bfloat16, device=DEV)
    torch.ops.fdl.softmax_argmax(logits, tok, prob)
    return tok, prob


@pytest.mark.parametrize("rows,vocab,scale", [(512, 152064, 2.0), (512, 152064, 0.3), (96, 151936, 1.0),
                                              (64, 1001, 0.05), (33, 8, 1.0)])
def test_softmax_argmax_vs_oracle_and_torch(rows, vocab, scale):
    g = torch.Generator(device=DEV).manual_seed(rows + vocab)
    pad = (vocab + 7) // 8 * 8  # rows 16-byte aligned; the logits are a [rows, :vocab] view
    base = (torch.randn(rows, pad, generator=g, device=DEV) * scale).to(torch.bfloat16)
    logits = base[:, :vocab]
    tok, prob = _fused(logits)
    et, ep = O.softmax_argmax_bf16(bits_of(logits))
    assert np.array_equal(tok.cpu().numpy(), et)
    assert np.abs(bits_of(prob).astype(np.int32) - ep.astype(np.int32)).max() <= 1
    p = torch.softmax(logits, dim=-1)
    x1 = p.argmax(-1)
    assert torch.equal(tok, x1)
    diff = (prob.view(torch.int16).int() - torch.gather(p, -1, x1[:, None])[:, 0].view(torch.int16).int()).abs()
    assert int(diff.max()) <= 1


def test_softmax_argmax_ties_and_3d_rows():
    logits = torch.zeros(2, 3, 4096, dtype=torch.bfloat16, device=DEV)
    logits[0, 0, 100] = logits[0, 0, 50] = 3.0
    logits[0, 1, 4095] = 1.0
    logits[1, 2, 7:30] = 0.001  # equal bf16 probabilities -> first index
    tok, prob = _fused(logits)
    et, ep = O.softmax_argmax_bf16(bits_of(logits.view(6, 4096)))
    assert tok.cpu().numpy().tolist() == et.tolist()
    assert tok.cpu().numpy().tolist()[:2] == [50, 4095]
    assert torch.equal(tok, torch.softmax(logits, -1).argmax(-1).view(-1))


def test_softmax_argmax_row_without_finite_logit_reports():
    logits = torch.full((2, 64), float("-inf"), dtype=torch.bfloat16, device=DEV)
    logits[0, 5] = 0.0
    tok, _ = _fused(logits)
    code, info = _lib.last_device_error()
    assert code == 1 and info == 1
    assert tok.cpu().tolist() == [5, 0]
