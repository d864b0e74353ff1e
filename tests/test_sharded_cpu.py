"""Row-sharded pair stack on CPU: shard plan, all-to-all transpose and the
full block orchestration against the single-device oracle
(``oracle/pairformer_oracle.py:pair_block``), on thread-emulated ranks and on
real ``gloo`` process groups (world size 2 and 3, the latter with an empty
rank), followed by the single stack on each rank's query rows. Phase math comes from ``tests/sharded_util.OraclePhases`` (float64),
so the comparison isolates the orchestration: tolerance 1e-10.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from fireprot_b200 import sharded as S
from oracle import pairformer_oracle as O

from sharded_util import OraclePhases, oracle_weight_dicts, run_threads, single_weight_dict

TOL = 1e-10


def test_shard_plan_covers_rows_once():
    for n in (1, 7, 31, 32, 33, 100, 1536, 3072):
        for w in (1, 2, 3, 4, 8):
            shards = [S.shard_plan(n, w, r) for r in range(w)]
            assert all(s.chunk % 32 == 0 and s.chunk * w >= n for s in shards)
            covered = []
            for s in shards:
                assert s.r0 == min(s.rank * s.chunk, n)
                covered.extend(range(s.r0, s.r0 + s.rows))
            assert covered == list(range(n))
    assert S.shard_plan(1536, 8, 3).rows == 192
    with pytest.raises(ValueError):
        S.shard_plan(10, 2, 2)


@pytest.mark.parametrize("n,world", [(40, 2), (70, 3), (33, 4), (33, 8)])
def test_transpose_rows_threads(n, world):
    z = torch.randn(n, n, 6, dtype=torch.float64, generator=torch.Generator().manual_seed(n))

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        zt = S.transpose_rows(S.local_rows(z, sh), sh, comm)
        assert torch.equal(zt[:sh.rows], z.transpose(0, 1)[sh.r0:sh.r0 + sh.rows])
        assert not zt[sh.rows:].any()
        back = S.transpose_rows(zt, sh, comm)
        assert torch.equal(back[:sh.rows], z[sh.r0:sh.r0 + sh.rows])
        S.transpose_rows(zt, sh, comm, out=zt)  # in place
        assert torch.equal(zt[:sh.rows], z[sh.r0:sh.r0 + sh.rows])
        return S.gather_rows(S.local_rows(z, sh), sh, comm)

    for full in run_threads(world, rank_fn):
        assert torch.equal(full, z)


def _case(n, mask_kind, seed=3):
    z = O.make_pair(n, seed=seed, dtype=torch.float64)
    p = O.make_block_params(seed=seed + 1, dtype=torch.float64)
    if mask_kind == "none":
        mask = None
    elif mask_kind == "padding":
        mask = O.make_padding_mask(n, n - 5, dtype=torch.float64)
    else:
        g = torch.Generator().manual_seed(seed + 2)
        mask = (torch.rand(n, n, generator=g) > 0.2).double()
    return z, mask, p


def _sharded_block(z, mask, p, rank, comm):
    sh = S.shard_plan(z.shape[0], comm.world, rank)
    z_loc = S.local_rows(z, sh)
    phases = OraclePhases()
    S.sharded_pair_block(z_loc, mask, oracle_weight_dicts(p), sh, comm, phases)
    return S.gather_rows(z_loc, sh, comm), phases.calls


@pytest.mark.parametrize("n,world,mask_kind", [(40, 1, "none"), (40, 2, "padding"),
                                               (70, 3, "random"), (45, 4, "padding")])
def test_sharded_block_threads(n, world, mask_kind):
    z, mask, p = _case(n, mask_kind)
    ref = O.pair_block(z, mask, p)
    outs = run_threads(world, lambda r, comm: _sharded_block(z, mask, p, r, comm))
    for full, calls in outs:
        assert O.rel_max_err(full, ref) <= TOL
        assert calls.count("trimul_finish") == 2 and calls.count("triattn_finish") == 2


def _sharded_full_block(z, s, mask, p, ps, rank, comm):
    """Whole Pairformer block: the sharded pair stack, then the single stack
    on the rank's query rows with s all-gathered after it."""
    sh = S.shard_plan(z.shape[0], comm.world, rank)
    z_loc = S.local_rows(z, sh)
    phases = OraclePhases()
    S.sharded_pair_block(z_loc, mask, oracle_weight_dicts(p), sh, comm, phases)
    s_buf = S.single_buffer(s, sh)
    S.sharded_single_block(s_buf, z_loc, mask, single_weight_dict(ps), sh, comm, phases)
    return S.gather_rows(z_loc, sh, comm), s_buf[:sh.n].clone(), phases.calls


def _full_ref(z, s, mask, p, ps):
    z1 = O.pair_block(z, mask, p)
    return z1, O.single_block(s, z1, mask, ps)


@pytest.mark.parametrize("n,world,mask_kind", [(40, 1, "padding"), (45, 2, "random"),
                                               (70, 3, "none"), (33, 4, "padding")])
def test_sharded_full_block_threads(n, world, mask_kind):
    z, mask, p = _case(n, mask_kind)
    s = O.make_single(n, seed=n, dtype=torch.float64)
    ps = O.make_single_params(seed=7, dtype=torch.float64, ln_affine_random=True)
    z_ref, s_ref = _full_ref(z, s, mask, p, ps)
    outs = run_threads(world, lambda r, comm: _sharded_full_block(z, s, mask, p, ps, r, comm))
    for z_full, s_full, calls in outs:
        assert O.rel_max_err(z_full, z_ref) <= TOL
        assert O.rel_max_err(s_full, s_ref) <= TOL
        assert calls.count("single_block") == 1


@pytest.mark.parametrize("outgoing", [True, False])
def test_sharded_trimul_add_false_threads(outgoing):
    n, world = 50, 2
    z, mask, p = _case(n, "random")
    ref = O.triangle_multiplication(z, mask, p.tri_mul_out, outgoing=outgoing, add=False)
    w = oracle_weight_dicts(p)["tri_mul_out"]

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        z_loc = S.local_rows(z, sh)
        S.sharded_trimul(z_loc, mask, w, sh, comm, OraclePhases(), outgoing=outgoing, add=False)
        return S.gather_rows(z_loc, sh, comm)

    for full in run_threads(world, rank_fn):
        assert O.rel_max_err(full, ref) <= TOL


@pytest.mark.parametrize("n,world,scheme", [(50, 2, "channels"), (45, 4, "channels"),
                                            (45, 4, "rows"), (33, 8, "channels"),
                                            (70, 8, "channels")])
@pytest.mark.parametrize("outgoing", [True, False])
def test_sharded_trimul_schemes_threads(n, world, scheme, outgoing):
    """Both exchange schemes of the TriMul contraction, including ranks with
    ragged and empty row ranges (n=33 over 8 ranks: 32 + 1 + six empty)."""
    z, mask, p = _case(n, "random")
    w = oracle_weight_dicts(p)["tri_mul_out" if outgoing else "tri_mul_in"]
    ref = O.triangle_multiplication(z, mask, p.tri_mul_out if outgoing else p.tri_mul_in,
                                    outgoing=outgoing, add=True)

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        z_loc = S.local_rows(z, sh)
        ph = OraclePhases()
        S.sharded_trimul(z_loc, mask, w, sh, comm, ph, outgoing=outgoing, scheme=scheme)
        return S.gather_rows(z_loc, sh, comm), ph.calls

    for full, calls in run_threads(world, rank_fn):
        assert O.rel_max_err(full, ref) <= TOL
        assert ("trimul_contract_groups" in calls) == (scheme == "channels")


def test_trimul_scheme_choice():
    assert [S.trimul_scheme(w) for w in (1, 2, 3, 4, 5, 6, 8, 16)] == \
        ["rows", "rows", "rows", "channels", "rows", "rows", "channels", "channels"]
    assert [S.trimul_scheme(w, "peer") for w in (1, 2, 3, 4, 5, 8)] == \
        ["rows", "channels", "rows", "channels", "rows", "channels"]
    z, mask, p = _case(40, "none")
    sh = S.shard_plan(40, 3, 0)
    with pytest.raises(ValueError):
        S.sharded_trimul(S.local_rows(z, sh), mask, oracle_weight_dicts(p)["tri_mul_out"], sh,
                         None, OraclePhases(), outgoing=True, scheme="channels")
    with pytest.raises(ValueError):
        S.sharded_trimul(S.local_rows(z, sh), mask, oracle_weight_dicts(p)["tri_mul_out"], sh,
                         None, OraclePhases(), outgoing=True, scheme="columns")


# ----------------------------------------------------------------- gloo ranks
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, n, mask_kind, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        z, mask, p = _case(n, mask_kind)
        s = O.make_single(n, seed=n, dtype=torch.float64)
        ps = O.make_single_params(seed=7, dtype=torch.float64)
        z_full, s_full, _ = _sharded_full_block(z, s, mask, p, ps, rank, S.DistComm())
        torch.save((z_full, s_full), os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,world,mask_kind", [(40, 2, "padding"), (40, 3, "random"),
                                               (70, 4, "random")])
def test_sharded_block_gloo(tmp_path, n, world, mask_kind):
    mp.start_processes(_gloo_rank, args=(world, _free_port(), n, mask_kind, str(tmp_path)),
                       nprocs=world, start_method="spawn")
    z, mask, p = _case(n, mask_kind)
    s = O.make_single(n, seed=n, dtype=torch.float64)
    z_ref, s_ref = _full_ref(z, s, mask, p, O.make_single_params(seed=7, dtype=torch.float64))
    for r in range(world):
        z_full, s_full = torch.load(tmp_path / f"rank{r}.pt")
        assert O.rel_max_err(z_full, z_ref) <= TOL
        assert O.rel_max_err(s_full, s_ref) <= TOL
