"""Multi-rank host logic on CPU: tile partitioning and the output gather, with gloo ranks
(world size 2 and 3), plus a rank that fails before the gather (the others must see an error,
not hang)."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest

from jasnamacos_b200.sharding import shard_range

REPO = Path(__file__).resolve().parent.parent


def test_shard_range_covers_every_tile_once():
    for total in (0, 1, 7, 128, 2048):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (b0, e0), (b1, _) in zip(ranges, ranges[1:]):
                assert e0 == b1
            sizes = [e - b for b, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, per_tile, fail_rank, q, mode="gather", chunks=3):
    sys.path.insert(0, str(REPO))
    import datetime

    import torch
    import torch.distributed as dist

    from jasnamacos_b200.sharding import compute_and_gather, gather_to_root, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        b, e = shard_range(total, rank, world)
        local = torch.arange(b * per_tile, e * per_tile, dtype=torch.float32)  # "output" of my tiles
        if rank == fail_rank:
            raise RuntimeError("injected host-side failure before the gather")
        if mode == "gather":
            full = gather_to_root(local, total, per_tile, dist)
        else:  # chunks computed into place and sent to rank 0 as they finish
            computed = []

            def compute(cb, ce, dst):
                computed.append((cb, ce))
                dst.copy_(torch.arange(cb * per_tile, ce * per_tile, dtype=torch.float32))

            full = torch.full((total * per_tile,), -1.0) if rank == 0 else None
            mine = torch.empty((e - b) * per_tile) if rank != 0 else None
            for w in compute_and_gather(compute, total, per_tile, dist, local=mine, full=full, chunks=chunks):
                w.wait()
            assert sum(ce - cb for cb, ce in computed) == e - b
            if rank != 0:
                assert torch.equal(mine, local)
                full = None
        if rank == 0:
            q.put(("ok", bool(torch.equal(full, torch.arange(total * per_tile, dtype=torch.float32)))))
        else:
            q.put(("ok", full is None))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put(("error", f"{rank}: {type(exc).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, total, per_tile, fail_rank=-1, timeout=60, mode="gather", chunks=3):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, per_tile, fail_rank, q, mode, chunks))
             for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for _ in range(world):
        results.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world,total", [(2, 7), (3, 16)])
def test_gather_to_root_gloo(world, total):
    results = _run(world, total, per_tile=5)
    assert all(kind == "ok" and flag for kind, flag in results), results


def test_failed_rank_surfaces_as_error_not_hang():
    results = _run(2, 8, per_tile=3, fail_rank=1, timeout=90)
    kinds = sorted(kind for kind, _ in results)
    assert kinds == ["error", "error"], results  # rank 1 failed; rank 0's recv timed out or was aborted


@pytest.mark.parametrize("world,total,chunks", [(2, 7, 3), (3, 16, 4), (3, 2, 4)])
def test_compute_and_gather_gloo(world, total, chunks):
    """The overlapped pass: every rank computes its shard chunk by chunk and each finished
    chunk is sent to rank 0 (some chunks empty when a shard is shorter than the chunk count)."""
    results = _run(world, total, per_tile=5, mode="pipelined", chunks=chunks)
    assert all(kind == "ok" and flag for kind, flag in results), results


def test_pipeline_chunks_and_root_share():
    from jasnamacos_b200.sharding import chunk_ranges, pipeline_chunks, root_share_for_ingress

    assert pipeline_chunks(0, 245, 4, 15) == [(0, 15)] + chunk_ranges(15, 245, 4)
    assert pipeline_chunks(10, 20, 4) == chunk_ranges(10, 20, 4)
    assert pipeline_chunks(10, 20, 2, 10) == chunk_ranges(10, 20, 2)  # first chunk not shorter than the range
    for b, e, c, f in [(0, 245, 4, 15), (7, 8, 3, 1), (100, 356, 8, 16)]:
        plan = pipeline_chunks(b, e, c, f)
        assert plan[0][0] == b and plan[-1][1] == e
        assert all(plan[i][1] == plan[i + 1][0] for i in range(len(plan) - 1))
    # Root's compute ends when the ingress of the others' tiles (after their first chunk) does.
    tc, ti = 3.45e-6, 0.655e-6
    share = root_share_for_ingress(2048, 8, tc, ti, first=16)
    r = share * 2048
    assert abs(r * tc - (16 * tc + (2048 - r) * ti)) < 1e-9
    assert root_share_for_ingress(2048, 8, 1.0, 1e-6) == 1.0 / 8  # fast links: never below the even share
    assert root_share_for_ingress(16, 2, 1e-6, 1.0) > 0.999  # slow links: root keeps (almost) everything
    assert root_share_for_ingress(16, 2, 1.0, 1.0, first=16) == 1.0  # capped at the whole batch


def test_weighted_ranges_and_sample_tiles():
    from jasnamacos_b200.sharding import chunk_ranges, sample_tiles, weighted_ranges

    for total, world, share in ((2048, 8, 0.19), (2048, 2, 0.1), (7, 3, 0.5), (100, 4, 1.0)):
        ranges = weighted_ranges(total, world, 0, share)
        assert ranges[0][0] == 0 and ranges[-1][1] == total
        assert all(e0 == b1 for (_, e0), (b1, _) in zip(ranges, ranges[1:]))
        assert ranges[0][1] - ranges[0][0] >= total // world  # root never below its even share
        rest = [e - b for b, e in ranges[1:]]
        assert max(rest) - min(rest) <= 1
    assert weighted_ranges(2048, 8, 0, 0.19)[0] == (0, 389)
    assert chunk_ranges(256, 512, 4) == [(256, 320), (320, 384), (384, 448), (448, 512)]
    s = sample_tiles(2048, 8, 16)
    assert len(s) == 128 and s[0] == 0 and s[-1] == 2047 and 255 in s and 256 in s
    assert sample_tiles(128, 8, 2) == [0, 15, 16, 31, 32, 47, 48, 63, 64, 79, 80, 95, 96, 111, 112, 127]
