"""Multi-rank host logic on CPU ranks (gloo, world_size 2): sharding covers every unit exactly
once, sharded oracle results gathered over the process group equal the unsharded ones, and a
rank that fails on the host ends its peer's collective with an error instead of a hang."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelforge_b200.shard import batch_head_shard, contiguous_range, row_shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_contiguous_ranges_partition_units():
    for units in (0, 1, 7, 8, 140, 262144):
        for world in (1, 2, 3, 8):
            spans = [contiguous_range(units, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == units
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    pairs = [p for r in range(8) for p in batch_head_shard(2, 70, 8, r)]
    assert pairs == [(b, h) for b in range(2) for h in range(70)]
    with pytest.raises(ValueError):
        contiguous_range(4, 2, 2)


def _worker(rank, world, port, mode, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    timeout = datetime.timedelta(seconds=5 if mode == "fail" else 60)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
    try:
        if mode == "gather":
            from oracle.rmsnorm import rmsnorm_forward

            g = torch.Generator().manual_seed(0)
            x = torch.randn(37, 96, generator=g)
            w = 1 + 0.1 * torch.randn(96, generator=g)
            mine = rmsnorm_forward(x[row_shard(37, world, rank)], w, 1e-6)
            sizes = [row_shard(37, world, r).stop - row_shard(37, world, r).start for r in range(world)]
            padded = torch.zeros(max(sizes), 96)
            padded[: mine.shape[0]] = mine
            gathered = [torch.zeros_like(padded) for _ in range(world)]
            dist.all_gather(gathered, padded)
            full = torch.cat([gathered[r][: sizes[r]] for r in range(world)])
            t = torch.tensor([float(rank + 1)])
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            queue.put((rank, bool(torch.equal(full, rmsnorm_forward(x, w, 1e-6))), float(t)))
        else:
            if rank == 1:
                raise RuntimeError("injected host failure before the collective")
            t = torch.ones(1)
            try:
                dist.all_reduce(t)
                queue.put((rank, "completed"))
            except Exception as exc:  # the peer never joined: the group timeout ends the wait
                queue.put((rank, f"error: {type(exc).__name__}"))
    except RuntimeError as exc:
        queue.put((rank, f"raised: {exc}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    results = [queue.get(timeout=5) for _ in range(2)]
    return {r[0]: r[1:] for r in results}


def test_sharded_rows_gather_to_the_unsharded_result():
    out = _run("gather")
    assert out[0][0] and out[1][0]
    assert out[0][1] == 2.0 and out[1][1] == 2.0  # max over ranks


def test_host_failure_ends_peer_collective_with_error():
    out = _run("fail")
    assert out[1][0].startswith("raised")
    assert out[0][0].startswith("error"), out[0]
