"""World-size-2 gloo tests of the multi-GPU host logic, on CPU.

Covers the token sharding (every row owned exactly once, 9914 -> 1240/1239
on 8 ranks), the column-parallel all-gather reassembly, max-over-ranks
timing, and host-side failure detection: a rank that raises before a
collective makes the other rank's collective fail with an error within the
process group's short timeout instead of hanging.
"""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from m5kernels_b200 import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _worker_gather(rank, world, port, out_q):
    try:
        _init(rank, world, port)
        m, n = 5, 8
        full = torch.arange(m * n, dtype=torch.float32).reshape(m, n)
        c0, c1 = sharding.shard_columns(n, world, rank)
        got = sharding.gather_columns(full[:, c0:c1].clone(), world)
        ms = sharding.max_over_ranks(1.0 + rank)
        r0, r1 = sharding.shard_rows(9914, world, rank)
        out_q.put((rank, torch.equal(got, full), ms, (r0, r1)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, repr(e), None, None))


def _worker_fail(rank, world, port, out_q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("injected host-side failure before the collective")
        t = torch.ones(4)
        dist.all_reduce(t)
        out_q.put((rank, "no error"))
    except RuntimeError as e:
        out_q.put((rank, "error: " + str(e)[:200]))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, "error: " + repr(e)[:200]))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_shard_rows_partition():
    for m in (0, 1, 7, 4096, 9914):
        for world in (1, 2, 4, 8):
            spans = [sharding.shard_rows(m, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == m
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert [b - a for a, b in (sharding.shard_rows(9914, 8, r) for r in range(8))] == [1240] * 2 + [1239] * 6
    with pytest.raises(ValueError):
        sharding.shard_rows(10, 2, 2)
    with pytest.raises(ValueError):
        sharding.shard_columns(10, 3, 0)


def test_gloo_two_ranks_gather_and_max():
    res = _run(_worker_gather)
    assert [r[1] for r in res] == [True, True], res
    assert [r[2] for r in res] == [2.0, 2.0]
    assert res[0][3] == (0, 4957) and res[1][3] == (4957, 9914)


def test_gloo_rank_failure_is_reported_not_hung():
    res = _run(_worker_fail, timeout=90)
    assert res[1][1].startswith("error: injected")
    assert res[0][1].startswith("error"), res
