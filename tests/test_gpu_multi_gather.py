"""GPU, two or more devices: the overlapped multi-GPU pass with the gather to rank 0.

Two ranks (one process per GPU, NCCL) each convolve their shard of a config-4-like batch chunk
by chunk; every finished chunk reaches rank 0 either over NCCL point-to-point
(sharding.compute_and_gather) or as a copy-engine peer copy into rank 0's tensor through a CUDA
IPC mapping (sharding.PeerGather + compute_and_copy_to_root), with even shards or with rank 0
taking a larger share in one chunk and the others starting with a short chunk.  Rank 0 must end up with exactly
the output a single dcn_forward_f16 call over the whole batch gives on its own GPU.  Skipped
when fewer than two GPUs are visible.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    sys.path.insert(0, str(REPO))
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from jasnamacos_b200 import sharding, synthetic
        from jasnamacos_b200.deform_conv import CudaDeformConv

        op = CudaDeformConv(rank)
        total, seed = 40, 5
        full_shape = synthetic.config_shape(4, batch=total)
        x, off, msk, w, b = synthetic.device_batch(full_shape, 16.0, seed=seed, device="cuda")
        w16 = torch.from_numpy(w).cuda().half()
        b16 = torch.from_numpy(b).cuda().half()
        packed = op.prepack(full_shape, w16)
        one = full_shape.with_batch(1)
        per = one.output_count
        lo, hi = sharding.shard_range(total, rank, world)
        mine = op.forward_f16(full_shape.with_batch(hi - lo), x[lo * one.input_count:hi * one.input_count],
                              off[lo * one.offset_count:hi * one.offset_count],
                              msk[lo * one.mask_count:hi * one.mask_count], packed, b16) if rank else None
        ref = op.forward_f16(full_shape, x, off, msk, packed, b16) if rank == 0 else None

        def compute(cb, ce, dst):
            op.forward_f16(one.with_batch(ce - cb), x[cb * one.input_count:ce * one.input_count],
                           off[cb * one.offset_count:ce * one.offset_count],
                           msk[cb * one.mask_count:ce * one.mask_count], packed, b16, out=dst)

        # Root-weighted layout (rank 0 takes 70% of the images in one chunk, the other ranks start
        # with a five-image chunk): the ranges differ from shard_range.  Every chunk keeps at least
        # three 64x64 images (96 tiles), so no chunk takes the group split and every image's bits
        # are those of the single call.
        weighted = sharding.weighted_ranges(total, world, 0, 0.7)
        wlo, whi = weighted[rank]
        mine_w = op.forward_f16(full_shape.with_batch(whi - wlo), x[wlo * one.input_count:whi * one.input_count],
                                off[wlo * one.offset_count:whi * one.offset_count],
                                msk[wlo * one.mask_count:whi * one.mask_count], packed, b16) if rank else None
        results = {}
        for mode in ("nccl", "peer", "peer_weighted"):
            full = torch.full((total * per,), float("nan"), dtype=torch.float16, device="cuda") if rank == 0 else None
            n_local = (whi - wlo) if mode == "peer_weighted" else (hi - lo)
            local = torch.empty(n_local * per, dtype=torch.float16, device="cuda") if rank else None
            if mode == "nccl":
                for wk in sharding.compute_and_gather(compute, total, per, dist, local=local, full=full, chunks=3):
                    wk.wait()
            else:
                peer = sharding.PeerGather(full, total, per, dist)
                if mode == "peer":
                    sharding.compute_and_copy_to_root(compute, total, per, dist, peer, local=local, full=full,
                                                      chunks=3)
                else:
                    sharding.compute_and_copy_to_root(compute, total, per, dist, peer, local=local, full=full,
                                                      chunks=1, ranges=weighted, first_chunk=5, root_chunks=1)
                torch.cuda.synchronize()
                dist.barrier()
                peer.close()
                dist.barrier()
            torch.cuda.synchronize()
            dist.barrier()
            if rank == 0:
                results[mode] = bool(torch.equal(full, ref))
            else:
                results[mode] = bool(torch.equal(local, mine_w if mode == "peer_weighted" else mine))
        q.put(("ok", rank, results))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put(("error", rank, f"{type(exc).__name__}: {exc}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_overlapped_gather_two_gpus():
    import multiprocessing as mp

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(kind == "ok" for kind, _, _ in out), out
    for _, rank, res in out:
        assert res == {"nccl": True, "peer": True, "peer_weighted": True}, (rank, res)
