"""Multi-rank host logic of bench.py on CPU with the gloo backend (world size 2): batch
sharding covers every row once, the job time is the max over ranks, and a rank that dies
before a collective makes the survivor fail with an error within the process-group
timeout instead of hanging."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def test_shard_covers_every_row_once():
    for total in (1, 2, 15, 16, 17):
        for world in (1, 2, 3, 4, 8):
            rows = []
            for r in range(world):
                start, n = bench.shard(total, world, r)
                rows += list(range(start, start + n))
            assert rows == list(range(total)), (total, world)
    with pytest.raises(ValueError):
        bench.shard(16, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "max":
            out = bench.max_over_ranks([float(rank), 10.0 - rank], dist)
            q.put((rank, out))
        elif mode == "dead":
            if rank == 1:
                os._exit(3)  # dies before the collective, without cleanup
            try:
                bench.max_over_ranks([1.0], dist)
                q.put((rank, "no error"))
            except Exception as e:  # gloo reports the lost peer or the timeout
                q.put((rank, "error: " + type(e).__name__))
    finally:
        if mode != "dead":
            dist.destroy_process_group()


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda t: t[0]), [p.exitcode for p in procs]


def test_max_over_ranks_gloo():
    out, codes = _run("max")
    assert codes == [0, 0]
    assert [o[1] for o in out] == [[1.0, 10.0], [1.0, 10.0]]


def test_dead_rank_gives_error_not_hang():
    out, codes = _run("dead")
    assert codes[1] == 3
    assert out and out[0][0] == 0 and out[0][1].startswith("error"), out
