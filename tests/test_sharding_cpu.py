"""Multi-process host logic of the sequence-sharded path on CPU (gloo,
world size 2): shard ranges, the final all-gather of generated ids, the
max-over-ranks timing reduction, and a rank that fails before the collective
(the other rank's collective ends with an error within the group timeout)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fast_v2_b200.sharding import gather_generated, max_over_ranks, sequence_shard


def test_sequence_shard_covers_all_sequences_once():
    for total in (0, 1, 7, 64, 129):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                first, n = sequence_shard(total, world, r)
                seen.extend(range(first, first + n))
            assert seen == list(range(total))
    with pytest.raises(ValueError):
        sequence_shard(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if mode == "ok":
            first, n = sequence_shard(5, world, rank)
            toks = torch.arange(first, first + n, dtype=torch.int64)[:, None] * 100 + torch.arange(3 + rank)
            full = gather_generated(toks, pad_id=-1)
            t = max_over_ranks(10.0 + rank)
            out_q.put((rank, full.tolist(), t))
        else:
            if rank == 1:
                os._exit(3)  # this rank dies before the collective
            try:
                gather_generated(torch.zeros(2, 4, dtype=torch.int64), pad_id=-1)
                out_q.put((rank, "no error", None))
            except Exception as e:  # noqa: BLE001 - any failure of the collective is the expected outcome
                out_q.put((rank, "error", type(e).__name__))
    finally:
        if mode == "ok":
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    n_reports = 2 if mode == "ok" else 1
    res = [q.get(timeout=120) for _ in range(n_reports)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    if mode != "ok":
        res.append((1, "exit" if procs[1].exitcode == 3 else f"exitcode {procs[1].exitcode}", None))
    return sorted(res, key=lambda r: r[0])


def test_gather_generated_and_max_over_ranks_world2():
    res = _run("ok")
    expected = [[0, 1, 2, -1], [100, 101, 102, -1], [200, 201, 202, -1], [300, 301, 302, 303],
                [400, 401, 402, 403]]
    for rank, full, t in res:
        assert full == expected
        assert t == 11.0


def test_rank_failure_surfaces_as_collective_error():
    res = _run("fail")
    assert res[1][1] == "exit"
    assert res[0][1] == "error"
