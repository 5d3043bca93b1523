"""Tile sharding across GPUs (one process per GPU).

The DCNv2 path partitions naturally: each output tile depends only on its own input,
offset and mask plus the replicated weights, so rank r of `world` processes a contiguous
range of tiles and there is no collective on the data path.  The one exchange the
production flow needs -- bringing every shard's output to one rank -- is
:func:`gather_to_root`, used after (never inside) a timed step.
"""

from __future__ import annotations


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Tiles [begin, end) of `rank`: contiguous, sizes differ by at most one, every tile once."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} rank={rank} world={world}")
    return total * rank // world, total * (rank + 1) // world


def gather_to_root(local, total_tiles: int, per_tile: int, dist, root: int = 0, out=None):
    """Collects every rank's shard of a [tiles * per_tile] output onto `root`.

    `local` is this rank's contiguous shard (a torch tensor); `dist` is
    torch.distributed with an initialised process group (NCCL for CUDA tensors, gloo for
    CPU).  Ranks exchange point-to-point (shards may differ in size by one tile); root posts
    all its receives in one batch, so the shards arrive concurrently (over NVLink for NCCL).
    `out` (root only, optional) receives the full tensor.  Returns the full tensor on root
    and None elsewhere.  Every rank takes the same steps.
    """
    import torch

    rank, world = dist.get_rank(), dist.get_world_size()
    b, e = shard_range(total_tiles, rank, world)
    if local.numel() != (e - b) * per_tile:
        raise ValueError("local shard has the wrong size")
    if rank != root:
        for req in dist.batch_isend_irecv([dist.P2POp(dist.isend, local.contiguous(), root)]):
            req.wait()
        return None
    full = out if out is not None else torch.empty(total_tiles * per_tile, dtype=local.dtype, device=local.device)
    if full.numel() != total_tiles * per_tile:
        raise ValueError("out has the wrong size")
    full[b * per_tile:e * per_tile].copy_(local)
    ops = []
    for src in range(world):
        if src == root:
            continue
        sb, se = shard_range(total_tiles, src, world)
        ops.append(dist.P2POp(dist.irecv, full[sb * per_tile:se * per_tile], src))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return full


def sample_tiles(total: int, ranges: int, per_range: int) -> list[int]:
    """A deterministic parity sample: `per_range` tile indices spread evenly over each of the
    `ranges` shard ranges of shard_range(total, r, ranges), first and last tile of every range
    included (fewer when a range is shorter)."""
    out: list[int] = []
    for r in range(ranges):
        b, e = shard_range(total, r, ranges)
        n = e - b
        if n <= 0:
            continue
        k = min(per_range, n)
        if k == 1:
            out.append(b)
            continue
        out.extend(sorted({b + (i * (n - 1)) // (k - 1) for i in range(k)}))
    return out


def chunk_ranges(begin: int, end: int, chunks: int) -> list[tuple[int, int]]:
    """`chunks` consecutive ranges covering [begin, end) (sizes differ by at most one; empty
    ranges allowed), the same split rule on every rank."""
    n = end - begin
    return [(begin + n * k // chunks, begin + n * (k + 1) // chunks) for k in range(chunks)]


def compute_and_gather(compute, total_tiles: int, per_tile: int, dist, local=None, full=None, root: int = 0,
                       chunks: int = 4):
    """One pass over this rank's tile shard with the gather to `root` overlapped: the shard is
    cut into `chunks` consecutive chunks (chunk_ranges, the same rule on every rank); after
    `compute(b, e, dst)` has enqueued chunk [b, e) (global tile indices) on the current
    stream, writing its output into `dst`, the chunk goes to `root` over NCCL point-to-point
    while the next chunk is computed.  NCCL's stream waits only for the work enqueued before
    the send, so the transfer of chunk k overlaps the kernels of chunk k+1.

    `local` (non-root ranks) is the rank's [shard * per_tile] output tensor; `full` (root) the
    [total_tiles * per_tile] tensor that receives every shard -- root computes its own chunks
    straight into it.  Returns the list of NCCL work handles; the caller waits on them
    (work.wait() orders the current stream after the transfers).  Every rank takes the same
    steps in the same order."""
    rank, world = dist.get_rank(), dist.get_world_size()
    b, e = shard_range(total_tiles, rank, world)
    mine = chunk_ranges(b, e, chunks)
    peers = {src: chunk_ranges(*shard_range(total_tiles, src, world), chunks) for src in range(world) if src != root}
    works = []
    for k, (cb, ce) in enumerate(mine):
        if rank == root:
            if ce > cb:
                compute(cb, ce, full[cb * per_tile:ce * per_tile])
            ops = [dist.P2POp(dist.irecv, full[pb * per_tile:pe * per_tile], src)
                   for src, ranges in peers.items() for pb, pe in [ranges[k]] if pe > pb]
        else:
            dst = local[(cb - b) * per_tile:(ce - b) * per_tile]
            if ce > cb:
                compute(cb, ce, dst)
            ops = [dist.P2POp(dist.isend, dst, root)] if ce > cb else []
        if ops:
            works.extend(dist.batch_isend_irecv(ops))
    return works
