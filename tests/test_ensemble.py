"""Member sharding and the output all-gather of mosaic_b200.ensemble, on CPU gloo
ranks (world size 2 and 3). Rank failure is made on the host: a rank that raises
before the collective must surface as an error on the others within the process
group timeout, never as a hang."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mosaic_b200 import ensemble as E


def test_member_range_partitions():
    for members in (1, 3, 24, 25):
        for world in (1, 2, 3, 8):
            got = [E.member_range(members, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == members
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    assert E.member_range(24, 2, 8) == (6, 9)


def test_noise_sharding_matches_full_draw():
    full = E.full_batch_noise(24, 32, "cpu")
    parts = [E.shard_rows(full, r, 8) for r in range(8)]
    assert torch.equal(torch.cat(parts), full)
    assert torch.equal(E.full_batch_noise(24, 32, "cpu"), full)  # same seed, same rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, members, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        full = torch.arange(members * 6, dtype=torch.float32).reshape(members, 2, 3)
        if mode == "fail" and rank == 1:
            raise RuntimeError("planted failure on rank 1 before the collective")
        out = E.run_sharded(lambda x: x * 2 + 1, [full], members)
        q.put((rank, "ok", torch.equal(out, full * 2 + 1)))
    except Exception as e:  # report instead of hanging the test
        q.put((rank, "error", repr(e)[:200]))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, members, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, members, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    res = {}
    while not q.empty():
        r, status, info = q.get()
        res[r] = (status, info)
    return res


@pytest.mark.parametrize("world,members", [(2, 24), (3, 7)])
def test_gather_on_gloo_ranks(world, members):
    res = _run(world, members, "ok")
    assert len(res) == world
    assert all(s == "ok" and info is True for s, info in res.values()), res


def test_rank_failure_is_an_error_not_a_hang():
    res = _run(2, 24, "fail")
    assert res[1][0] == "error"
    assert res[0][0] == "error"  # rank 0's collective times out / aborts with an error
