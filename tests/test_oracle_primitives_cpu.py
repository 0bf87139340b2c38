"""The oracle's copy and gather primitives against the torch ops the
reference calls for them, run on CPU tensors on random inputs (bit for bit):
scatter_ with repeated positions, slice-append at per-sequence starts,
cat + repeat_kv, gather along the sequence axis."""
import numpy as np
import torch

from oracle import kvcache_oracle as O


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _rand(shape, g):
    return torch.randn(*shape, generator=g).to(torch.bfloat16)


def test_scatter_rows_equals_torch_scatter_with_repeats():
    g = torch.Generator().manual_seed(1)
    B, S, H, D, n = 3, 40, 2, 16, 12
    for trial in range(10):
        dst = _rand((B, S, H, D), g)
        src = _rand((B, n, H, D), g)
        pos = torch.randint(0, S, (B, n), generator=g)
        pos[:, -1] = pos[:, 0]  # a repeated position in every row
        want = dst.clone().scatter_(1, pos[:, :, None, None].expand(B, n, H, D), src)
        got = O.scatter_rows(_bits(dst).copy(), _bits(src), pos.numpy())
        assert np.array_equal(got, _bits(want)), trial


def test_scatter_rows_bhsd_axis_equals_torch():
    g = torch.Generator().manual_seed(2)
    B, H, S, D, n = 2, 4, 32, 8, 5
    dst, src = _rand((B, H, S, D), g), _rand((B, H, n, D), g)
    pos = torch.stack([torch.randperm(S, generator=g)[:n] for _ in range(B)])
    want = dst.clone().scatter_(2, pos[:, None, :, None].expand(B, H, n, D), src)
    got = O.scatter_rows(_bits(dst).copy(), _bits(src), pos.numpy(), seq_axis=2)
    assert np.array_equal(got, _bits(want))


def test_append_at_per_sequence_starts_equals_write_sparse_positions():
    g = torch.Generator().manual_seed(3)
    B, S, H, D, n = 4, 64, 2, 8, 16
    kc, vc = _rand((B, S, H, D), g), _rand((B, S, H, D), g)
    k, v = _rand((B, n, H, D), g), _rand((B, n, H, D), g)
    start = torch.tensor([0, 5, 48, 17], dtype=torch.int32)
    pos = start[:, None].long() + torch.arange(n)[None, :]
    idx = pos[:, :, None, None].expand(B, n, H, D)
    wk, wv = kc.clone().scatter_(1, idx, k), vc.clone().scatter_(1, idx, v)
    ek, ev = O.kv_append(_bits(kc).copy(), _bits(vc).copy(), _bits(k), _bits(v), start.numpy())
    assert np.array_equal(ek, _bits(wk)) and np.array_equal(ev, _bits(wv))


def test_packed_prefix_gather_equals_cat_and_repeat_kv():
    g = torch.Generator().manual_seed(4)
    B, S, H, D, n, rep = 3, 50, 2, 8, 4, 7
    cache, block = _rand((B, S, H, D), g), _rand((B, n, H, D), g)
    lens = np.array([0, 17, 50], np.int32)
    got, cu = O.gather_prefix_packed(_bits(cache), lens, rep, _bits(block))
    parts = [torch.cat([cache[b, : lens[b]], block[b]], 0).repeat_interleave(rep, dim=1) for b in range(B)]
    assert np.array_equal(got, _bits(torch.cat(parts, 0)))
    assert cu.tolist() == [0, 4, 4 + 21, 4 + 21 + 54]


def test_gather_rows_equals_torch_gather():
    g = torch.Generator().manual_seed(5)
    B, S, H, n = 2, 30, 64, 9
    x = _rand((B, S, H), g)
    idx = torch.randint(0, S, (B, n), generator=g)
    want = x.gather(1, idx[:, :, None].expand(B, n, H))
    assert np.array_equal(O.gather_rows(_bits(x), idx.numpy()), _bits(want))
