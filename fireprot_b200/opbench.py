"""Per-operator device benchmark (the reference's operator A/B harness role,
``benchmarks/protenix/benchmark_triangle.py``).

  python -m fireprot_b200.opbench --op trimul_out --n 1024 --precision strict

Runs one operator (or the whole pair block) on a seeded synthetic pair tensor
``--iters`` times after ``--warmup`` runs and prints one JSON line with the
mean device time per call and the per-kernel device times (CUDA events around
every launch). Ops: trimul_out, trimul_in, triattn_start, triattn_end,
transition, block, packed_bmm, single (the single stack, s [n, 384]),
openfold3_attention (the OpenFold3 ``_attention`` scope on q, k, v
[n, 4, n, 32] with a [1, 1, 1, n] mask and a [1, 4, n, n] bias, i.e. one
triangle attention of an OpenFold3 trunk through the scope),
esm_contract_out / esm_contract_in (ESMFold2's channels-last triangle
contraction, [1, n, n, 256]).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops
from .modules import PairformerPairBlock


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="block")
    ap.add_argument("--n", type=int, default=1024)
    ap.add_argument("--precision", default="strict")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--mask", action="store_true", help="padding mask (valid = n - n/32)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    n = a.n
    g = torch.Generator().manual_seed(0)
    z = torch.randn(n, n, 128, generator=g).to(dev)
    mask = None
    if a.mask:
        v = torch.arange(n) < n - n // 32
        mask = (v[:, None] & v[None, :]).float().to(dev)
    blk = PairformerPairBlock().init_random_(1).to(dev)

    if a.op == "block":
        ws = ops.pair_block_workspace(n, a.precision, mask is not None, dev)
        cw = blk.c_weights()

        def run():
            ops.pair_block(z, mask, cw, precision=a.precision, workspace=ws)
    elif a.op in ("trimul_out", "trimul_in"):
        m = blk.tri_mul_out if a.op == "trimul_out" else blk.tri_mul_in

        def run():
            m(z, mask, precision=a.precision)
    elif a.op in ("triattn_start", "triattn_end"):
        m = blk.tri_att_start if a.op == "triattn_start" else blk.tri_att_end

        def run():
            m(z, mask, precision=a.precision)
    elif a.op == "transition":
        def run():
            blk.pair_transition(z, precision=a.precision)
    elif a.op == "single":
        from .modules import PairformerSingleBlock
        sblk = PairformerSingleBlock().init_random_(2).to(dev)
        s = torch.randn(n, 384, generator=g).to(dev)
        sws = ops.single_block_workspace(n, n, dev)
        cws = sblk.c_weights()

        def run():
            ops.single_block(s, z, mask, cws, precision=a.precision, workspace=sws)
    elif a.op == "openfold3_attention":
        from types import SimpleNamespace

        from . import backend
        from .openfold3 import AttentionCoreKernel, AttentionDispatcher, _scoped_hook
        backend.set_precision(a.precision)
        del z
        q = (torch.randn(n, 4, n, 32, generator=g) / 32 ** 0.5).to(dev)
        k = torch.randn(n, 4, n, 32, generator=g).to(dev)
        v = torch.randn(n, 4, n, 32, generator=g).to(dev)
        valid = (torch.arange(n) < n - n // 32).float()
        biases = [(1e9 * (valid - 1.0)).view(1, 1, 1, n).to(dev),
                  torch.randn(1, 4, n, n, generator=g).to(dev)]
        target = SimpleNamespace(_attention=None)
        disp = AttentionDispatcher(AttentionCoreKernel(0))

        def run():
            with torch.no_grad(), _scoped_hook(target, disp):
                target._attention(q, k, v, biases)
    elif a.op in ("esm_contract_out", "esm_contract_in"):
        del z
        lt = torch.randn(1, n, n, 256, generator=g).to(dev)
        rt = torch.randn(1, n, n, 256, generator=g).to(dev)

        def run():
            ops.triangle_contract(lt, rt, outgoing=a.op == "esm_contract_out",
                                  precision=a.precision)
    elif a.op == "packed_bmm":
        x = torch.randn(128, n, n, generator=g).to(dev)
        y = torch.randn(128, n, n, generator=g).to(dev)

        def run():
            ops.packed_bmm(x, y, True, a.precision)
    else:
        raise SystemExit(f"unknown op {a.op}")

    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize(dev)
    ops.timing_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    rec = ops.timing_collect()
    ops.timing_enable(False)
    print(json.dumps({"op": a.op, "n": n, "precision": a.precision,
                      "ms_per_call": e0.elapsed_time(e1) / a.iters,
                      "kernels": {k: {"launches": v["launches"],
                                      "avg_ms": v["total_ms"] / v["launches"]}
                                  for k, v in rec.items()}}))


if __name__ == "__main__":
    main()
