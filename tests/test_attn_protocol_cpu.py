"""A model of the block-attention kernel's barrier protocol
(fast_v2_b200/csrc/block_attn.cuh), run under random timing on the CPU.

The kernel's warps (TMA producer, MMA issuer, four softmax warps per 128-row
tile, some of them padding warps) hand work to each other through mbarriers
that complete after a fixed number of arrivals and are waited on by phase
parity; MMA completion reaches a barrier through a commit that fires when
every MMA issued before it has finished.  Timing decides which interleavings
happen on the GPU, and the GPU tests see only a few of them.  The model
replays the protocol of both pipelines -- one row tile (S double-buffered, P
in its own TMEM columns) and two row tiles (P over S, S(j+1) after P(j)*V_j)
-- with random latencies, from K/V tiles that arrive at once (L2-resident)
to slow ones, and checks: no wait that can never finish, every P*V_j issued
only after each computing warp wrote P(j), no S buffer rewritten before every
warp read it, and O rescaled only after the previous P*V completed.

It also shows why the padding warps of the one-tile pipeline take their
p_full turn only after P(j-1)*V_(j-1): without that gate, fast K/V tiles let
them arrive for tile j+1 before the other warps arrive for tile j.
"""
import random

import pytest


class _Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        return (self.phase & 1) != parity


class _Sim:
    def __init__(self, seed, tma):
        self.rnd = random.Random(seed)
        self.tma = tma
        self.bars = {}
        self.pending = []  # (finish, kind, tile, row_tile, id)
        self.commits = []
        self.issued = []
        self.now = 0
        self.next_id = 0
        self.errors = []
        self.state = {}

    def bar(self, name, count):
        self.bars[name] = _Bar(count)

    def mma(self, kind, j, m):
        i = self.next_id
        self.next_id += 1
        start = max([f for f, *_ in self.pending] + [self.now])
        self.pending.append((start + self.rnd.randint(5, 20), kind, j, m, i))
        self.issued.append(i)
        return i

    def complete(self, kind, j, m):
        return not any(k == kind and jj == j and mm == m for _, k, jj, mm, _ in self.pending)

    def commit(self, name):
        self.commits.append((name, {x[-1] for x in self.pending}))

    def wait(self, name, parity):
        while not self.bars[name].done(parity):
            yield

    def delay(self, lo, hi):
        for _ in range(self.rnd.randint(lo, hi)):
            yield

    def run(self, progs, limit=200000):
        alive = list(range(len(progs)))
        steps = 0
        while alive:
            steps += 1
            self.now += 1
            if steps > limit:
                return False
            self.pending = [p for p in self.pending if p[0] > self.now]
            live = {p[-1] for p in self.pending}
            for c in list(self.commits):
                if not (c[1] & live):
                    self.commits.remove(c)
                    self.bars[c[0]].arrive()
            self.rnd.shuffle(alive)
            for k in list(alive):
                try:
                    next(progs[k])
                except StopIteration:
                    alive.remove(k)
        return True


def _producer(sim, T):
    for j in range(T):
        st = j % 2
        if j >= 2:
            yield from sim.wait(f"kv_empty{st}", ((j // 2) - 1) & 1)
        yield from sim.delay(*sim.tma)
        sim.bars[f"kv_full{st}"].arrive()


def one_row_tile(seed, T, n_pad, tma, gate_padding=True):
    """n_mt == 1: S(j) in buffer j & 1, P in its own columns, 4 softmax warps
    of which the last n_pad hold only padding rows."""
    sim = _Sim(seed, tma)
    for name, c in [("kv_full0", 1), ("kv_full1", 1), ("kv_empty0", 1), ("kv_empty1", 1), ("s_full0", 1),
                    ("s_full1", 1), ("p_full", 4), ("pv_done", 1), ("s_free0", 4), ("s_free1", 4)]:
        sim.bar(name, c)
    wrote, read = set(), set()

    def issuer():
        yield from sim.wait("kv_full0", 0)
        sim.mma("S", 0, 0)
        sim.commit("s_full0")
        for j in range(T):
            if j + 1 < T:
                yield from sim.wait(f"kv_full{(j + 1) % 2}", ((j + 1) // 2) & 1)
                if j >= 1:
                    yield from sim.wait(f"s_free{(j + 1) & 1}", ((j - 1) >> 1) & 1)
                    if any((j - 1, w) not in read for w in range(4)):
                        sim.errors.append(f"S({j + 1}) overwrites S({j - 1}) before every warp read it")
                sim.mma("S", j + 1, 0)
                sim.commit(f"s_full{(j + 1) & 1}")
            yield from sim.wait("p_full", j & 1)
            if any((j, w) not in wrote for w in range(4 - n_pad)):
                sim.errors.append(f"P*V({j}) issued before every computing warp wrote P({j})")
            sim.mma("PV", j, 0)
            sim.commit("pv_done")
            if j + 2 < T:
                sim.commit(f"kv_empty{j % 2}")

    def softmax(w):
        pad = w >= 4 - n_pad
        for j in range(T):
            buf = j & 1
            yield from sim.wait(f"s_full{buf}", (j >> 1) & 1)
            if pad:
                read.add((j, w))
                sim.bars[f"s_free{buf}"].arrive()
                if gate_padding and j > 0:
                    yield from sim.wait("pv_done", (j - 1) & 1)
                sim.bars["p_full"].arrive()
                continue
            yield from sim.delay(3, 20)  # read S, row max
            if j > 0:
                yield from sim.wait("pv_done", (j - 1) & 1)  # P and O free
                if not sim.complete("PV", j - 1, 0):
                    sim.errors.append("O rescaled while P*V is in flight")
            yield from sim.delay(3, 20)  # lower half of P
            read.add((j, w))
            sim.bars[f"s_free{buf}"].arrive()
            yield from sim.delay(3, 20)  # upper half of P
            wrote.add((j, w))
            sim.bars["p_full"].arrive()
        yield from sim.wait("pv_done", (T - 1) & 1)

    ok = sim.run([_producer(sim, T), issuer()] + [softmax(w) for w in range(4)])
    return ok, sim.errors


def two_row_tiles(seed, T, pad_tile1, tma):
    """n_mt == 2: P_m(j) over S_m(j); S_m(j+1) issued after P_m(j)*V_j; the
    last pad_tile1 warps of row tile 1 hold only padding rows."""
    sim = _Sim(seed, tma)
    for name, c in [("kv_full0", 1), ("kv_full1", 1), ("kv_empty0", 1), ("kv_empty1", 1), ("s_full0", 1),
                    ("s_full1", 1), ("p_full0", 4), ("p_full1", 4), ("pv_done0", 1), ("pv_done1", 1)]:
        sim.bar(name, c)
    wrote = set()

    def pad(m, w):
        return m == 1 and w >= 4 - pad_tile1

    def issuer():
        yield from sim.wait("kv_full0", 0)
        for m in range(2):
            sim.mma("S", 0, m)
            sim.commit(f"s_full{m}")
        for j in range(T):
            for m in range(2):
                yield from sim.wait(f"p_full{m}", j & 1)
                if any((m, j, w) not in wrote for w in range(4) if not pad(m, w)):
                    sim.errors.append(f"P*V{m}({j}) issued before every computing warp wrote P")
                sim.mma("PV", j, m)
                sim.commit(f"pv_done{m}")
                if m == 1 and j + 2 < T:
                    sim.commit(f"kv_empty{j % 2}")
                if j + 1 < T:
                    if m == 0:
                        yield from sim.wait(f"kv_full{(j + 1) % 2}", ((j + 1) // 2) & 1)
                    yield from sim.wait(f"pv_done{m}", j & 1)
                    if not sim.complete("PV", j, m):
                        sim.errors.append(f"S{m}({j + 1}) over P{m}({j}) while P*V reads it")
                    sim.mma("S", j + 1, m)
                    sim.commit(f"s_full{m}")

    def softmax(m, w):
        for j in range(T):
            yield from sim.wait(f"s_full{m}", j & 1)
            if pad(m, w):
                sim.bars[f"p_full{m}"].arrive()
                continue
            if j > 0 and not sim.complete("PV", j - 1, m):
                sim.errors.append("O rescaled while P*V is in flight")
            yield from sim.delay(5, 40)
            wrote.add((m, j, w))
            sim.bars[f"p_full{m}"].arrive()
        yield from sim.wait(f"pv_done{m}", (T - 1) & 1)

    ok = sim.run([_producer(sim, T), issuer()] + [softmax(m, w) for m in range(2) for w in range(4)])
    return ok, sim.errors


TMA = [(1, 4), (1, 30), (60, 150)]  # K/V tiles from L2 at once ... slow HBM loads


@pytest.mark.parametrize("tma", TMA)
def test_one_row_tile_protocol(tma):
    for T in (1, 2, 3, 5, 8):
        for n_pad in (0, 1, 2, 3):
            for seed in range(25):
                ok, errors = one_row_tile(seed, T, n_pad, tma)
                assert ok, f"wait that never finishes: T={T} pad={n_pad} seed={seed}"
                assert not errors, (T, n_pad, seed, errors[:3])


@pytest.mark.parametrize("tma", TMA)
def test_two_row_tiles_protocol(tma):
    for T in (1, 2, 3, 5, 8):
        for pad_tile1 in (0, 1, 2):
            for seed in range(25):
                ok, errors = two_row_tiles(seed, T, pad_tile1, tma)
                assert ok, f"wait that never finishes: T={T} pad={pad_tile1} seed={seed}"
                assert not errors, (T, pad_tile1, seed, errors[:3])


def test_padding_warps_need_their_turn():
    """Without the gate, fast K/V tiles break the one-tile pipeline."""
    broken = 0
    for seed in range(40):
        ok, errors = one_row_tile(seed, 5, 2, (1, 4), gate_padding=False)
        broken += (not ok) or bool(errors)
    assert broken > 0
