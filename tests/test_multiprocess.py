"""The N > 1 host logic of bench.py on CPU: two `gloo` ranks.

Decode shards by request (sequences are independent): every rank takes a
contiguous, even block of the workload's sequences, runs them with no
data-path collective, and the job's time is the max over ranks.  These
tests run that logic as two processes with the gloo backend (127.0.0.1)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, total: int, q):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        first, count = bench.shard(total, world, rank)
        mine = torch.zeros(total, dtype=torch.int64)
        mine[first:first + count] = 1
        dist.all_reduce(mine)  # every sequence owned by exactly one rank
        # prompts are a function of the global sequence index only
        p = bench.prompts_for(first, count, (64, 960), 16384)
        ref = bench.prompts_for(0, total, (64, 960), 16384)[first:first + count]
        same = all((a == b).all() for a, b in zip(p, ref))
        # the job's time is the max over ranks
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tokens = torch.tensor([float(count * 7)], dtype=torch.float64)
        dist.all_reduce(tokens)
        q.put((rank, first, count, mine.tolist(), same, float(t.item()), float(tokens.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [64, 7, 1])
def test_request_sharding_over_two_gloo_ranks(total):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, f0, c0, own0, same0, t0, tok0), (r1, f1, c1, own1, same1, t1, tok1) = res
    assert own0 == [1] * total and own1 == own0
    assert f0 == 0 and f1 == c0 and c0 + c1 == total and abs(c0 - c1) <= 1
    assert same0 and same1
    assert t0 == t1 == 11.0
    assert tok0 == tok1 == 7.0 * total
