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

from kernelforge_b200.shard import batch_head_blocks, batch_head_shard, contiguous_range, row_shard


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


def test_batch_head_blocks_are_dense_rectangles_of_the_shard():
    for batch, heads, world in ((4, 36, 8), (2, 70, 8), (4, 16, 2), (2, 70, 3), (1, 70, 8), (3, 5, 4), (4, 16, 1)):
        for rank in range(world):
            blocks = batch_head_blocks(batch, heads, world, rank)
            assert len(blocks) <= 3
            units = [(b, h) for b0, b1, h0, h1 in blocks for b in range(b0, b1) for h in range(h0, h1)]
            assert units == batch_head_shard(batch, heads, world, rank)
            # A rectangle spanning several batches holds whole batches, so it is one dense slice.
            assert all(b1 - b0 == 1 or (h0, h1) == (0, heads) for b0, b1, h0, h1 in blocks)


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
        elif mode in ("blocks", "blocks_planted"):
            # bench.py's verification: each rank digests its (batch, head) blocks, rank 0 compares
            # them with the same slices of its unsharded result. The "planted" run changes one
            # element of rank 1's block on the CPU, which the comparison must report.
            os.environ.update(WORLD_SIZE=str(world), RANK=str(rank))
            import bench

            g = torch.Generator().manual_seed(5)
            x = torch.randn(3, 8, 5, 16, generator=g).to(torch.bfloat16)
            op = lambda t: (t.float() * 1.5 + 0.25).to(torch.bfloat16)  # noqa: E731
            mine = torch.zeros(3, 2, dtype=torch.int64)
            for j, blk in enumerate(batch_head_blocks(3, 5, world, rank)):
                out = op(bench.fa_block(x, blk))
                if mode == "blocks_planted" and rank == 1 and j == 0:
                    out.view(-1)[3] += 1
                mine[j] = bench.digest(out)

            def reference():
                full = op(x)
                refs = []
                for r in range(world):
                    ref = torch.zeros(3, 2, dtype=torch.int64)
                    for j, blk in enumerate(batch_head_blocks(3, 5, world, r)):
                        ref[j] = bench.digest(bench.fa_block(full, blk))
                    refs.append(ref)
                return refs

            res = bench.verify_digests(bench.Dist(), mine, reference)
            queue.put((rank, None if res is None else (res["ok"], res["mismatched_ranks"])))
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


def test_bench_verification_gathers_block_digests():
    out = _run("blocks")
    assert out[0][0] == (True, []) and out[1][0] is None
    planted = _run("blocks_planted")
    assert planted[0][0] == (False, [1])
