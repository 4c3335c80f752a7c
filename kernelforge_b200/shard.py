"""Sharding of the hot-path work across ranks (one process per GPU, no data-path collective).

Every operator here is independent along one axis: RMSNorm along rows, SANA attention along
(batch, head) pairs (its K^T V reduction stays inside a head), FlashAttention along
(batch, head). A rank's share is a contiguous range of that axis.
"""

from __future__ import annotations


def contiguous_range(units: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of ``rank``'s contiguous share of ``units`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world or units < 0:
        raise ValueError("need world > 0, 0 <= rank < world and units >= 0")
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def row_shard(rows: int, world: int, rank: int) -> slice:
    """Rows of an RMSNorm input that ``rank`` normalises."""
    start, stop = contiguous_range(rows, world, rank)
    return slice(start, stop)


def batch_head_shard(batch: int, heads: int, world: int, rank: int) -> list[tuple[int, int]]:
    """(batch, head) pairs of an attention problem that ``rank`` computes, in row-major order."""
    start, stop = contiguous_range(batch * heads, world, rank)
    return [divmod(u, heads) for u in range(start, stop)]


def batch_head_blocks(batch: int, heads: int, world: int, rank: int) -> list[tuple[int, int, int, int]]:
    """``rank``'s contiguous (batch, head) range as at most three rectangles
    ``(b_start, b_stop, h_start, h_stop)``: the tail of a first, partly owned batch, a run of whole
    batches, and the head of a last, partly owned batch. Each rectangle is one dense slice of a
    [batch, ..., heads, ...] tensor (SANA's packed qkv [B, N, 3, H*d], FlashAttention's
    [B, N, H, D]) and one kernel call."""
    start, stop = contiguous_range(batch * heads, world, rank)
    blocks = []
    u = start
    while u < stop:
        b, h = divmod(u, heads)
        if h == 0 and stop - u >= heads:
            nb = (stop - u) // heads
            blocks.append((b, b + nb, 0, heads))
            u += nb * heads
        else:
            h_stop = min(heads, h + (stop - u))
            blocks.append((b, b + 1, h, h_stop))
            u += h_stop - h
    return blocks
