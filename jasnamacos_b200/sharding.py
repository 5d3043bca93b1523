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


def pipeline_chunks(begin: int, end: int, chunks: int, first: int = 0) -> list[tuple[int, int]]:
    """[begin, end) cut for a compute + copy pipeline: a short first chunk of `first` tiles (so
    that the first copy starts early), then the rest in `chunks` near-equal chunks; without
    `first` (or when the range is no longer than it), chunk_ranges(begin, end, chunks)."""
    if 0 < first < end - begin:
        return [(begin, begin + first)] + chunk_ranges(begin + first, end, chunks)
    return chunk_ranges(begin, end, chunks)


def root_share_for_ingress(total: int, world: int, compute_s_per_tile: float, ingress_s_per_tile: float,
                           first: int = 0) -> float:
    """Share of the tiles for the root of a copy-engine gather such that its own compute ends
    when the others' outputs have arrived.  The root computes its R tiles in
    R * compute_s_per_tile; the others start copying after their first chunk (`first` tiles) and
    are then bound by the root's link ingress, (total - R) * ingress_s_per_tile.  Equal at
    R = (total * ingress + first * compute) / (compute + ingress); never below the even share."""
    r = (total * ingress_s_per_tile + first * compute_s_per_tile) / (compute_s_per_tile + ingress_s_per_tile)
    return min(1.0, max(1.0 / world, r / total))


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


class PeerGather:
    """Writes every rank's output chunks straight into one tensor on the root GPU with the
    copy engines (one cudaMemcpyAsync peer copy per chunk over NVLink), so no kernel and no SM
    time is spent on the transfer and it overlaps the next chunk's kernels completely.

    Root exports its full [total_tiles * per_tile] tensor through a CUDA IPC handle (plus the
    tensor's offset inside its allocation), every other rank opens it in its own device's
    address space.  `send` enqueues a chunk on the given stream; a copy is complete when that
    stream reaches the end of it.  `close` unmaps the handle on every rank (all ranks call it,
    followed by a barrier before root frees the tensor).  Host-side set-up uses the process group `dist` for the
    handle exchange; the transfers themselves use no collective."""

    def __init__(self, full, total_tiles: int, per_tile: int, dist, root: int = 0, element_size: int = 2):
        import torch
        from cuda.bindings import driver, runtime

        self._rt = runtime
        self.dist, self.root = dist, root
        self.rank = dist.get_rank()
        self.total_tiles, self.per_tile, self.es = total_tiles, per_tile, element_size
        dev = torch.device("cuda", torch.cuda.current_device())
        meta = torch.zeros(73, dtype=torch.uint8, device=dev)  # handle, offset, status byte
        self._mapped = None
        self.base = 0
        problem = None
        if self.rank == root:
            ptr = full.data_ptr()
            err, base, _size = driver.cuMemGetAddressRange(ptr)
            if err == driver.CUresult.CUDA_SUCCESS:
                err2, handle = runtime.cudaIpcGetMemHandle(int(base))
                if err2 == runtime.cudaError_t.cudaSuccess:
                    raw = bytes(handle.reserved) + int(ptr - int(base)).to_bytes(8, "little") + b"\x01"
                    meta.copy_(torch.frombuffer(bytearray(raw), dtype=torch.uint8))
                    self.base = ptr
                else:
                    problem = f"cudaIpcGetMemHandle failed: {err2}"
            else:
                problem = f"cuMemGetAddressRange failed: {err}"
        # Every rank takes this broadcast, also when root could not export its tensor.
        dist.broadcast(meta, src=root)
        raw = bytes(meta.cpu().tolist())
        if raw[72] != 1:
            raise RuntimeError(problem or "root could not export its output tensor")
        if self.rank != root:
            handle = runtime.cudaIpcMemHandle_t()
            handle.reserved = raw[:64]
            offset = int.from_bytes(raw[64:72], "little")
            err, mapped = runtime.cudaIpcOpenMemHandle(handle, runtime.cudaIpcMemLazyEnablePeerAccess)
            if err != runtime.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cudaIpcOpenMemHandle failed: {err}")
            self._mapped = int(mapped)
            self.base = self._mapped + offset

    def send(self, tile_begin: int, tile_end: int, src, stream) -> None:
        """Copies `src` (this rank's output of tiles [tile_begin, tile_end)) into root's tensor."""
        n = (tile_end - tile_begin) * self.per_tile * self.es
        if n == 0 or self.rank == self.root:
            return
        if src.numel() * src.element_size() != n:
            raise ValueError("chunk has the wrong size")
        dst = self.base + tile_begin * self.per_tile * self.es
        (err,) = self._rt.cudaMemcpyAsync(dst, src.data_ptr(), n, self._rt.cudaMemcpyKind.cudaMemcpyDefault,
                                          stream.cuda_stream)
        if err != self._rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"peer copy failed: {err}")

    def close(self) -> None:
        """Unmaps root's tensor on this rank (after this rank's copies are done).  Not a
        collective: the caller puts a barrier after every rank's close, before root frees."""
        import torch

        torch.cuda.synchronize()
        if self._mapped is not None:
            self._rt.cudaIpcCloseMemHandle(self._mapped)
            self._mapped = None


def weighted_ranges(total: int, world: int, root: int, root_share: float) -> list[tuple[int, int]]:
    """Contiguous tile ranges for every rank, `root` taking round(root_share * total) tiles (at
    least its even share) and the others splitting the rest evenly.  When the gather into root
    is limited by root's NVLink ingress rather than by compute, root should compute more: its
    own tiles never cross the link."""
    own = max(total // world, min(total, int(round(root_share * total))))
    rest = total - own
    others = [r for r in range(world) if r != root]
    sizes = {root: own}
    for i, r in enumerate(others):
        sizes[r] = rest * (i + 1) // len(others) - rest * i // len(others)
    out, b = [], 0
    for r in range(world):
        out.append((b, b + sizes[r]))
        b += sizes[r]
    return out


def compute_and_copy_to_root(compute, total_tiles: int, per_tile: int, dist, peer: PeerGather, local=None,
                             full=None, root: int = 0, chunks: int = 4, copy_stream=None, ranges=None,
                             first_chunk: int = 0, root_chunks: int | None = None):
    """compute_and_gather with the transfers made by the copy engines (PeerGather): after
    `compute(b, e, dst)` has enqueued chunk [b, e) on the current stream, `copy_stream` waits for
    it and copies the chunk into root's tensor while the current stream goes on with the next
    chunk.  At the end the current stream waits for the copy stream, so an event recorded after
    this call completes when this rank's outputs are all in root's memory.  `ranges` (one
    (begin, end) per rank, e.g. weighted_ranges) replaces the even shard_range split; the other
    ranks cut their range with pipeline_chunks(..., chunks, first_chunk), root (whose outputs do
    not move) into `root_chunks` chunks (default `chunks`)."""
    import torch

    rank, world = dist.get_rank(), dist.get_world_size()
    b, e = ranges[rank] if ranges is not None else shard_range(total_tiles, rank, world)
    cur = torch.cuda.current_stream()
    copy_stream = copy_stream or torch.cuda.Stream()
    plan = (chunk_ranges(b, e, root_chunks or chunks) if rank == root
            else pipeline_chunks(b, e, chunks, first_chunk))
    for cb, ce in plan:
        if ce <= cb:
            continue
        if rank == root:
            compute(cb, ce, full[cb * per_tile:ce * per_tile])
            continue
        dst = local[(cb - b) * per_tile:(ce - b) * per_tile]
        compute(cb, ce, dst)
        copy_stream.wait_stream(cur)
        peer.send(cb, ce, dst, copy_stream)
    cur.wait_stream(copy_stream)
