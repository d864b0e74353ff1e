"""Per-phase device-time split of the row-sharded Pairformer block.

  python -m torch.distributed.run --nnodes=1 --nproc-per-node 4 \\
      --master-addr 127.0.0.1 --master-port 29500 -m fireprot_b200.shardprof --comm peer

One process per GPU. Runs ``sharded_pair_block`` + ``sharded_single_block``
on a seeded N = 1536 pair tensor (padding mask, valid 1480) for a few
blocks, with CUDA events on the launch stream around every phase-kernel
call (``CudaPhases``) and every exchange call of the transport (``DistComm``
or ``PeerComm``), and prints one JSON line per rank from rank 0: the last
block's time and the summed device time of each call kind. The events sit
between the calls only, so the kernels themselves run as in ``bench.py``.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from . import sharded as S
from .modules import PairformerBlock


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", choices=["peer", "nccl"], default="peer")
    ap.add_argument("--n", type=int, default=1536)
    ap.add_argument("--valid", type=int, default=1480)
    ap.add_argument("--precision", choices=["strict", "fast"], default="strict")
    ap.add_argument("--blocks", type=int, default=4)
    a = ap.parse_args(argv)
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    n = a.n
    g = torch.Generator().manual_seed(1000)
    z_full = torch.randn(n, n, 128, generator=g)
    s = torch.randn(n, 384, generator=g)
    keep = torch.arange(n) < a.valid
    mask = (keep[:, None] & keep[None, :]).float().to(dev)
    block = PairformerBlock().init_random_(1).to(dev)
    shard = S.shard_plan(n, world, rank)
    comm = S.PeerComm() if a.comm == "peer" else S.DistComm()
    weights = S.block_weight_dicts(block.pair)
    w_single = block.single.weight_dict()
    z = S.local_rows(z_full, shard).to(dev)
    del z_full
    sbuf = S.single_buffer(s.to(dev), shard)
    phases = S.CudaPhases(a.precision)
    stream = torch.cuda.current_stream(dev)
    rec = []

    def timed(fn, label):
        def wrapper(*args, **kw):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            out = fn(*args, **kw)
            e1.record(stream)
            rec.append((label, e0, e1))
            return out
        return wrapper

    for name in ("all_gather", "reduce_scatter", "all_to_all", "transpose_rows", "barrier"):
        if hasattr(comm, name):
            setattr(comm, name, timed(getattr(comm, name), "comm." + name))
    for name in dir(phases):
        if name.startswith("_") or name in ("check", "trimul_group_plane"):
            continue
        if callable(getattr(phases, name)):
            setattr(phases, name, timed(getattr(phases, name), "phase." + name))
    try:
        for _ in range(a.blocks):
            rec.clear()
            dist.barrier()
            torch.cuda.synchronize(dev)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            S.sharded_pair_block(z, mask, weights, shard, comm, phases)
            S.sharded_single_block(sbuf, z, mask, w_single, shard, comm, phases)
            t1.record(stream)
            torch.cuda.synchronize(dev)
        phases.check()
        totals = {}
        for label, e0, e1 in rec:
            totals[label] = totals.get(label, 0.0) + e0.elapsed_time(e1)
        line = {"rank": rank, "world": world, "comm": a.comm, "precision": a.precision, "n": n,
                "block_ms": round(t0.elapsed_time(t1), 3),
                "ms": {k: round(v, 3) for k, v in sorted(totals.items())}}
        got = [None] * world
        dist.all_gather_object(got, line)
        if rank == 0:
            for item in got:
                print(json.dumps(item), flush=True)
        torch.cuda.synchronize(dev)
    finally:
        if isinstance(comm, S.PeerComm):
            torch.cuda.synchronize(dev)
            comm.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
