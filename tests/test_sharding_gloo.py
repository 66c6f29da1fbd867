"""Row sharding and the weight broadcast, as two gloo ranks on the CPU."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from triton_ops.sharding import RowShard, broadcast_tensors, shard_positions, shard_rows, slab_tables


def test_shard_rows_cover_exactly_once():
    for total in (0, 1, 7, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            shards = [shard_rows(total, world, r) for r in range(world)]
            assert shards[0].start == 0 and shards[-1].stop == total
            for a, b in zip(shards, shards[1:]):
                assert a.stop == b.start
            sizes = [s.rows for s in shards]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_slab_tables_positions():
    seq = 8
    cos = torch.arange(seq * 4, dtype=torch.float32).view(seq, 4)
    sin = -cos
    # whole sequences: tables unchanged
    c, s, b, sl = slab_tables(cos, sin, RowShard(1, 2, 16, 32), seq)
    assert c is cos and b == 2 and sl == seq
    # ragged slab: positions gathered, one long sequence
    sh = RowShard(0, 3, 5, 13)
    c, s, b, sl = slab_tables(cos, sin, sh, seq)
    assert (b, sl) == (1, 8)
    assert torch.equal(c[:, 0], cos[shard_positions(sh, seq), 0])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = torch.full((4, 3), float(rank + 1))
        t = torch.full((5,), float(rank + 10))
        broadcast_tensors([w, t], src=0)
        sh = shard_rows(10, world, rank)
        q.put((rank, w.sum().item(), t.sum().item(), sh.start, sh.stop))
    finally:
        dist.destroy_process_group()


def test_weight_broadcast_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res[0][1:3] == (12.0, 50.0) and res[1][1:3] == (12.0, 50.0)
    assert (res[0][3], res[0][4], res[1][3], res[1][4]) == (0, 5, 5, 10)


def _failing_worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves before the broadcast, with nothing in flight
    try:
        broadcast_tensors([torch.zeros(4)], src=0)
        q.put((rank, "no-error"))
    except Exception as e:  # the surviving rank must see an error, not hang
        q.put((rank, type(e).__name__))


def test_rank_failure_before_broadcast_is_reported():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    rank, outcome = q.get(timeout=30)
    assert rank == 0 and outcome != "no-error"
