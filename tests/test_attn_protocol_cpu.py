"""A model of the block-attention kernel's barrier protocol
(fast_v2_b200/csrc/block_attn.cuh), run under random timing on the CPU.

The kernel's warps (TMA producer, MMA issuer, four softmax warps per 128-row
tile, some of them padding warps) hand work to each other through mbarriers
that complete after a fixed number of arrivals and are waited on by phase
parity; MMA completion reaches a barrier through a commit that fires when
every MMA issued before it has finished.  Timing decides which interleavings
happen on the GPU, and the GPU tests see only a few of them.  The model
replays the protocol of both pipelines -- one row tile (S double-buffered, P
in its own TMEM columns) and two row tiles (P over S, S(j+1) queued right
behind P(j)*V_j: the tensor core runs one thread's MMAs in issue order, as the
model does) -- with random latencies, from K/V tiles that arrive at once (L2-resident)
to slow ones, and checks: no wait that can never finish, every P*V_j issued
only after each computing warp wrote P(j), no S buffer rewritten before every
warp read it (nor before the P*V that reads P out of it has finished), and O
rescaled only after the previous P*V completed.

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
        self.ids = {}
        self.start = {}
        self.finish = {}

    def bar(self, name, count):
        self.bars[name] = _Bar(count)

    def mma(self, kind, j, m):
        i = self.next_id
        self.next_id += 1
        start = max([f for f, *_ in self.pending] + [self.now])
        fin = start + self.rnd.randint(5, 20)
        self.pending.append((fin, kind, j, m, i))
        self.issued.append(i)
        self.ids[(kind, j, m)] = i
        self.start[i], self.finish[i] = start, fin
        return i

    def runs_after(self, i, kind, j, m):
        """MMA i starts only once the MMA (kind, j, m) has finished."""
        return self.finish[self.ids[(kind, j, m)]] <= self.start[i]

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
    """n_mt == 2: P_m(j) over S_m(j); S_m(j+1) queued right behind P_m(j)*V_j;
    the last pad_tile1 warps of row tile 1 hold only padding rows."""
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
                    i = sim.mma("S", j + 1, m)
                    if not sim.runs_after(i, "PV", j, m):
                        sim.errors.append(f"S{m}({j + 1}) over P{m}({j}) while P*V reads it")
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


# ---------------------------------------------------------------------------
# Persistent form: one CTA walks several work items (sequence x KV head x
# query chunk x split) with per-CTA running tile counters, so every per-tile
# barrier keeps its phase sequence across items.  Per item: the producer
# reloads Q only after the previous item's last S MMA (q_empty, a commit);
# the issuer waits q_full before the item's first S; the softmax warps do the
# item's epilogue (read O after its last P*V) before they take part in the
# next item's tiles, which is what lets the next item's first P*V (the one
# that overwrites O) follow from p_full alone.  Items may hold no tiles.
# ---------------------------------------------------------------------------


def _persistent_producer(sim, units):
    gt = nq = 0
    for T in units:
        if T == 0:
            continue
        if nq > 0:
            yield from sim.wait("q_empty", (nq - 1) & 1)
        if sim.state.get("S_in_flight")():
            sim.errors.append(f"Q of item {nq} loaded while an S MMA of the previous item is in flight")
        yield from sim.delay(*sim.tma)
        sim.bars["q_full"].arrive()
        for _ in range(T):
            st = gt % 2
            if gt >= 2:
                yield from sim.wait(f"kv_empty{st}", ((gt // 2) - 1) & 1)
            yield from sim.delay(*sim.tma)
            sim.bars[f"kv_full{st}"].arrive()
            gt += 1
        nq += 1


def persistent_two_row_tiles(seed, units, pad_tile1, tma):
    sim = _Sim(seed, tma)
    for name, c in [("kv_full0", 1), ("kv_full1", 1), ("kv_empty0", 1), ("kv_empty1", 1), ("s_full0", 1),
                    ("s_full1", 1), ("p_full0", 4), ("p_full1", 4), ("pv_done0", 1), ("pv_done1", 1),
                    ("q_full", 1), ("q_empty", 1)]:
        sim.bar(name, c)
    total = sum(units)
    wrote, o_read = set(), set()
    sim.state["S_in_flight"] = lambda: any(k == "S" for _, k, *_ in sim.pending)

    def pad(m, w):
        return m == 1 and w >= 4 - pad_tile1

    def issuer():
        gt = nq = 0
        for T in units:
            if T == 0:
                continue
            g0 = gt
            yield from sim.wait("q_full", nq & 1)
            yield from sim.wait(f"kv_full{g0 % 2}", (g0 // 2) & 1)
            for m in range(2):
                if g0 > 0:
                    yield from sim.wait(f"pv_done{m}", (g0 - 1) & 1)
                sim.mma("S", g0, m)
                sim.commit(f"s_full{m}")
            if T == 1:
                sim.commit("q_empty")
            for j in range(T):
                g = g0 + j
                for m in range(2):
                    yield from sim.wait(f"p_full{m}", g & 1)
                    if any((m, g, w) not in wrote for w in range(4) if not pad(m, w)):
                        sim.errors.append(f"P*V{m}({g}) issued before every computing warp wrote P")
                    if j == 0 and nq > 0 and any((nq - 1, m, w) not in o_read for w in range(4)):
                        sim.errors.append(f"first P*V{m} of item {nq} overwrites O before the epilogue read it")
                    sim.mma("PV", g, m)
                    sim.commit(f"pv_done{m}")
                    if m == 1 and g + 2 < total:
                        sim.commit(f"kv_empty{g % 2}")
                    if j + 1 < T:
                        if m == 0:
                            yield from sim.wait(f"kv_full{(g + 1) % 2}", ((g + 1) // 2) & 1)
                        i = sim.mma("S", g + 1, m)
                        if not sim.runs_after(i, "PV", g, m):
                            sim.errors.append(f"S{m}({g + 1}) over P{m}({g}) while P*V reads it")
                        sim.commit(f"s_full{m}")
                        if m == 1 and j + 1 == T - 1:
                            sim.commit("q_empty")
            gt += T
            nq += 1

    def softmax(m, w):
        gt = nq = 0
        for T in units:
            if T == 0:
                continue
            for j in range(T):
                g = gt + j
                yield from sim.wait(f"s_full{m}", g & 1)
                if pad(m, w):
                    sim.bars[f"p_full{m}"].arrive()
                    continue
                if j > 0 and not sim.complete("PV", g - 1, m):
                    sim.errors.append("O rescaled while P*V is in flight")
                yield from sim.delay(5, 40)
                wrote.add((m, g, w))
                sim.bars[f"p_full{m}"].arrive()
            yield from sim.wait(f"pv_done{m}", (gt + T - 1) & 1)  # epilogue: O of this item
            if not sim.complete("PV", gt + T - 1, m):
                sim.errors.append("epilogue read O before the item's last P*V completed")
            yield from sim.delay(2, 15)
            o_read.add((nq, m, w))
            gt += T
            nq += 1

    progs = [_persistent_producer(sim, units), issuer()] + [softmax(m, w) for m in range(2) for w in range(4)]
    ok = sim.run(progs)
    return ok, sim.errors


def persistent_one_row_tile(seed, units, n_pad, tma):
    sim = _Sim(seed, tma)
    for name, c in [("kv_full0", 1), ("kv_full1", 1), ("kv_empty0", 1), ("kv_empty1", 1), ("s_full0", 1),
                    ("s_full1", 1), ("p_full", 4), ("pv_done", 1), ("s_free0", 4), ("s_free1", 4),
                    ("q_full", 1), ("q_empty", 1)]:
        sim.bar(name, c)
    total = sum(units)
    wrote, read, o_read = set(), set(), set()
    sim.state["S_in_flight"] = lambda: any(k == "S" for _, k, *_ in sim.pending)

    def issue_s(g):
        if g >= 2:
            yield from sim.wait(f"s_free{g & 1}", ((g - 2) >> 1) & 1)
            if any((g - 2, w) not in read for w in range(4)):
                sim.errors.append(f"S({g}) overwrites S({g - 2}) before every warp read it")
        sim.mma("S", g, 0)
        sim.commit(f"s_full{g & 1}")

    def issuer():
        gt = nq = 0
        for T in units:
            if T == 0:
                continue
            g0 = gt
            yield from sim.wait("q_full", nq & 1)
            yield from sim.wait(f"kv_full{g0 % 2}", (g0 // 2) & 1)
            yield from issue_s(g0)
            if T == 1:
                sim.commit("q_empty")
            for j in range(T):
                g = g0 + j
                if j + 1 < T:
                    yield from sim.wait(f"kv_full{(g + 1) % 2}", ((g + 1) // 2) & 1)
                    yield from issue_s(g + 1)
                    if j + 1 == T - 1:
                        sim.commit("q_empty")
                yield from sim.wait("p_full", g & 1)
                if any((g, w) not in wrote for w in range(4 - n_pad)):
                    sim.errors.append(f"P*V({g}) issued before every computing warp wrote P({g})")
                if j == 0 and nq > 0 and any((nq - 1, w) not in o_read for w in range(4)):
                    sim.errors.append(f"first P*V of item {nq} overwrites O before the epilogue read it")
                sim.mma("PV", g, 0)
                sim.commit("pv_done")
                if g + 2 < total:
                    sim.commit(f"kv_empty{g % 2}")
            gt += T
            nq += 1

    def softmax(w):
        pad = w >= 4 - n_pad
        gt = nq = 0
        for T in units:
            if T == 0:
                continue
            for j in range(T):
                g = gt + j
                buf = g & 1
                yield from sim.wait(f"s_full{buf}", (g >> 1) & 1)
                if pad:
                    read.add((g, w))
                    sim.bars[f"s_free{buf}"].arrive()
                    if g > 0:
                        yield from sim.wait("pv_done", (g - 1) & 1)
                    sim.bars["p_full"].arrive()
                    continue
                yield from sim.delay(3, 20)
                if g > 0:
                    yield from sim.wait("pv_done", (g - 1) & 1)  # P (and, within the item, O) free
                    if not sim.complete("PV", g - 1, 0):
                        sim.errors.append("P rewritten while P*V is in flight")
                yield from sim.delay(3, 20)
                read.add((g, w))
                sim.bars[f"s_free{buf}"].arrive()
                yield from sim.delay(3, 20)
                wrote.add((g, w))
                sim.bars["p_full"].arrive()
            yield from sim.wait("pv_done", (gt + T - 1) & 1)
            if not sim.complete("PV", gt + T - 1, 0):
                sim.errors.append("epilogue read O before the item's last P*V completed")
            yield from sim.delay(2, 15)
            o_read.add((nq, w))
            gt += T
            nq += 1

    ok = sim.run([_persistent_producer(sim, units), issuer()] + [softmax(w) for w in range(4)])
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


UNITS = [[3], [1, 1], [2, 0, 3], [1, 4, 2], [0, 2, 1, 1], [5, 5], [1, 0, 0, 1]]


@pytest.mark.parametrize("tma", TMA)
def test_persistent_two_row_tiles_protocol(tma):
    for units in UNITS:
        for pad_tile1 in (0, 2):
            for seed in range(15):
                ok, errors = persistent_two_row_tiles(seed, units, pad_tile1, tma)
                assert ok, f"wait that never finishes: items={units} pad={pad_tile1} seed={seed}"
                assert not errors, (units, pad_tile1, seed, errors[:3])


@pytest.mark.parametrize("tma", TMA)
def test_persistent_one_row_tile_protocol(tma):
    for units in UNITS:
        for n_pad in (0, 2):
            for seed in range(15):
                ok, errors = persistent_one_row_tile(seed, units, n_pad, tma)
                assert ok, f"wait that never finishes: items={units} pad={n_pad} seed={seed}"
                assert not errors, (units, n_pad, seed, errors[:3])
