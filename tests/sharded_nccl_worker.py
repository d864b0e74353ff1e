"""torchrun worker for ``test_gpu_sharded_nccl.py``: one process per GPU,
NCCL process group, the whole Pairformer block on each rank's rows (the
sharded pair stack, then the single stack on the rank's query rows and the
all-gather of s), then rank 0 compares the all-gathered z and s with the CPU
oracle and writes a JSON verdict to ``argv[1]``, over NCCL collectives and
over the peer-memory transport. Every rank runs the same collective
sequence."""
import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from fireprot_b200 import sharded as S  # noqa: E402
from oracle import pairformer_oracle as O  # noqa: E402
from sharded_util import oracle_weight_dicts, single_weight_dict  # noqa: E402


def main(out_path: str) -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    comms = {"nccl": S.DistComm(), "peer": S.PeerComm()}
    comm = comms["nccl"]
    results = {}
    try:
        for n, mask_kind in ((150, "padding"), (96, "none")):
            z = O.make_pair(n, seed=71 + n)
            mask = O.make_padding_mask(n, n - 9) if mask_kind == "padding" else None
            p = O.make_block_params(seed=17)
            w = {k: {kk: (None if vv is None else vv.to(dev)) for kk, vv in d.items()}
                 for k, d in oracle_weight_dicts(p).items()}
            md = None if mask is None else mask.to(dev)
            s = O.make_single(n, seed=n)
            ps = O.make_single_params(seed=19, ln_affine_random=True)
            ws = {k: v.to(dev) for k, v in single_weight_dict(ps).items()}
            sh = S.shard_plan(n, comm.world, comm.rank)
            ref = O.pair_block(z, mask, p) if comm.rank == 0 else None
            s_ref = O.single_block(s, ref, mask, ps) if comm.rank == 0 else None
            # both TriMul exchange schemes at every world size (the channel
            # scheme is the default only from four ranks)
            # and both transports (NCCL collectives, peer-memory copies)
            for precision, scheme, kind in (("strict", "rows", "nccl"), ("fast", "rows", "nccl"),
                                            ("strict", "channels", "nccl"),
                                            ("fast", "channels", "nccl"),
                                            ("strict", "rows", "peer"),
                                            ("strict", "channels", "peer"),
                                            ("fast", "channels", "peer")):
                comm = comms[kind]
                z_loc = S.local_rows(z.to(dev), sh)
                s_buf = S.single_buffer(s.to(dev), sh)
                ph = S.CudaPhases(precision)
                S.sharded_pair_block(z_loc, md, w, sh, comm, ph, scheme=scheme)
                S.sharded_single_block(s_buf, z_loc, md, ws, sh, comm, ph)
                torch.cuda.synchronize(dev)
                ph.check()
                full = S.gather_rows(z_loc, sh, comm).cpu()
                if comm.rank == 0:
                    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
                    err = O.rel_max_err(full, ref)
                    err_s = O.rel_max_err(s_buf[:n].cpu(), s_ref)
                    results[f"n{n}_{mask_kind}_{precision}_{scheme}_{kind}"] = {
                        "err": err, "err_s": err_s, "tol": tol,
                        "ok": err <= tol and err_s <= tol}
        dist.barrier()
        torch.cuda.synchronize(dev)
    finally:
        comms["peer"].close()
        dist.destroy_process_group()
    if comm.rank == 0:
        Path(out_path).write_text(json.dumps({"world": comm.world, "cases": results}))


if __name__ == "__main__":
    main(sys.argv[1])
