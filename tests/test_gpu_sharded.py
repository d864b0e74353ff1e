"""GPU parity of the row-sharded phase kernels (``fpb_trimul_shard_*``,
``fpb_triattn_shard_*``) against the single-device oracle.

Ranks are emulated by threads on one GPU (``sharded_util.ThreadComm``: the
collectives are tensor copies between the threads' buffers, every launch on
one stream), so each rank's kernels run on its own row range, including
ragged and empty ranks. The NCCL path itself is covered by
``test_gpu_sharded_nccl.py``. Tolerances: strict 1e-4, fast 1e-2 of the
fp32 output scale (single operators); the full block accumulates five
updates, and is held to the same bounds.
"""
import pytest
import torch

from fireprot_b200 import sharded as S
from oracle import pairformer_oracle as O

from sharded_util import oracle_weight_dicts, run_threads

pytestmark = pytest.mark.gpu


def _dev(d, device):
    return {k: (None if v is None else v.to(device)) for k, v in d.items()}


def _tol(precision):
    return O.STRICT_TOL if precision == "strict" else O.FAST_TOL


def _mask(n, kind):
    if kind == "none":
        return None
    if kind == "padding":
        return O.make_padding_mask(n, n - 7)
    g = torch.Generator().manual_seed(11)
    return (torch.rand(n, n, generator=g) > 0.25).float()


def _run(world, n, z, mask, device, body):
    md = None if mask is None else mask.to(device)

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        z_loc = S.local_rows(z.to(device), sh)
        phases = body(z_loc, md, sh, comm)
        torch.cuda.synchronize(device)
        phases.check()
        return S.gather_rows(z_loc, sh, comm).cpu()

    return run_threads(world, rank_fn)


@pytest.mark.parametrize("world,n,scheme", [(2, 100, "rows"), (3, 70, "rows"), (4, 40, "rows"),
                                            (2, 100, "channels"), (4, 200, "channels"),
                                            (8, 33, "channels"), (8, 300, "channels")])
@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_sharded_trimul(cuda_device, world, n, scheme, outgoing, precision):
    z = O.make_pair(n, seed=21 + n)
    mask = _mask(n, "random")
    p = O.make_trimul_params(seed=5, ln_affine_random=True)
    ref = O.triangle_multiplication(z, mask, p, outgoing=outgoing, add=True)
    w = _dev({k: getattr(p, k) for k in ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p",
                                         "w_b_g", "w_g", "ln_out_w", "ln_out_b", "w_z")},
             cuda_device)

    def body(z_loc, md, sh, comm):
        ph = S.CudaPhases(precision)
        S.sharded_trimul(z_loc, md, w, sh, comm, ph, outgoing=outgoing, scheme=scheme)
        return ph

    for full in _run(world, n, z, mask, cuda_device, body):
        assert O.rel_max_err(full, ref) <= _tol(precision)


@pytest.mark.parametrize("world,n", [(2, 100), (3, 70)])
@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
@pytest.mark.parametrize("mask_kind", ["none", "padding"])
def test_sharded_triattn(cuda_device, world, n, starting, precision, mask_kind):
    z = O.make_pair(n, seed=31 + n)
    mask = _mask(n, mask_kind)
    p = O.make_triattn_params(seed=9)
    ref = z + O.triangle_attention(z, mask, p, starting=starting)
    w = _dev({k: getattr(p, k) for k in ("ln_w", "ln_b", "w_q", "w_k", "w_v", "w_bias", "w_g",
                                         "b_g", "w_o", "b_o")}, cuda_device)

    def body(z_loc, md, sh, comm):
        ph = S.CudaPhases(precision)
        S.sharded_triattn(z_loc, md, w, sh, comm, ph, starting=starting)
        return ph

    for full in _run(world, n, z, mask, cuda_device, body):
        assert O.rel_max_err(full, ref) <= _tol(precision)


@pytest.mark.parametrize("world,n,mask_kind", [(1, 96, "padding"), (2, 150, "padding"),
                                               (3, 100, "none"), (5, 130, "random"),
                                               (4, 130, "random"), (8, 260, "padding")])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_sharded_block(cuda_device, world, n, mask_kind, precision):
    z = O.make_pair(n, seed=41 + n)
    mask = _mask(n, mask_kind)
    p = O.make_block_params(seed=13)
    ref = O.pair_block(z, mask, p)
    w = {k: _dev(v, cuda_device) for k, v in oracle_weight_dicts(p).items()}

    def body(z_loc, md, sh, comm):
        ph = S.CudaPhases(precision)
        S.sharded_pair_block(z_loc, md, w, sh, comm, ph)
        return ph

    for full in _run(world, n, z, mask, cuda_device, body):
        assert O.rel_max_err(full, ref) <= _tol(precision)


@pytest.mark.parametrize("count", [1, 7, 4096, 100003])
@pytest.mark.parametrize("in_place", [False, True])
def test_split_tf32_exact(cuda_device, count, in_place):
    """``fpb_split_tf32``: hi has the low 13 mantissa bits clear and
    hi + lo reproduces every FP32 input exactly (also in place)."""
    from fireprot_b200 import _lib
    g = torch.Generator().manual_seed(count)
    x = (torch.randn(count, generator=g) * torch.exp(torch.randn(count, generator=g) * 4)).to(
        cuda_device)
    src = x.clone()
    hi = src if in_place else torch.empty_like(x)
    lo = torch.empty_like(x)
    lib = _lib.load()
    assert lib.fpb_split_tf32(src.data_ptr(), hi.data_ptr(), lo.data_ptr(), count,
                              torch.cuda.current_stream(cuda_device).cuda_stream) == 0
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(hi.view(torch.int32) & 0x1FFF, torch.zeros_like(hi, dtype=torch.int32))
    assert torch.equal((hi.double() + lo.double()), x.double())


@pytest.mark.parametrize("cols_mode", [0, 1])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_group_gather_exact(cuda_device, cols_mode, precision):
    """``fpb_trimul_group_gather``: the stacked (rows) or concatenated (cols)
    reorder of a received [world][G][rows][ld] block, bit-exact against the
    same torch reorder, with the strict hi/lo split of every element."""
    from fireprot_b200 import _lib
    W, G, R, ld, seg = 4, 8, 40, 64, (64 if cols_mode == 0 else 32)
    dt = torch.float32 if precision == "strict" else torch.bfloat16
    g = torch.Generator().manual_seed(5 + cols_mode)
    src = torch.randn(W, G, R, ld, generator=g).to(dt).to(cuda_device)
    if cols_mode == 0:
        ref = src[..., :seg].transpose(0, 1).reshape(G, W * R, seg)
        dst_rows, dst_ld = W * R, ld
    else:
        ref = src[..., :seg].permute(1, 2, 0, 3).reshape(G, R, W * seg)
        dst_rows, dst_ld = R, W * seg + 4
    hi = torch.full((G, dst_rows, dst_ld), 7.0, dtype=dt, device=cuda_device)
    lo = torch.full_like(hi, 7.0) if precision == "strict" else None
    lib = _lib.load()
    assert lib.fpb_trimul_group_gather(
        src.data_ptr(), W, G, R, ld, seg, cols_mode, hi.data_ptr(),
        0 if lo is None else lo.data_ptr(), dst_ld, 0 if precision == "strict" else 1,
        torch.cuda.current_stream(cuda_device).cuda_stream) == 0
    torch.cuda.synchronize(cuda_device)
    width = ref.shape[-1]
    assert torch.all(hi[..., width:] == 7.0)  # nothing written past the operand
    if precision == "strict":
        got_hi, got_lo = hi[..., :width], lo[..., :width]
        assert torch.equal(got_hi.view(torch.int32) & 0x1FFF,
                           torch.zeros_like(got_hi, dtype=torch.int32))
        assert torch.equal(got_hi.double() + got_lo.double(), ref.double())
    else:
        assert torch.equal(hi[..., :width], ref)


@pytest.mark.parametrize("world,n,mask_kind", [(2, 100, "random"), (3, 70, "padding"),
                                               (5, 40, "none")])
def test_sharded_single_block(cuda_device, world, n, mask_kind):
    """Single stack on each rank's query rows, then the all-gather of s."""
    from sharded_util import single_weight_dict
    s = O.make_single(n, seed=71 + n)
    z = O.make_pair(n, seed=72 + n)
    mask = _mask(n, mask_kind)
    p = O.make_single_params(seed=23, ln_affine_random=True)
    ref = O.single_block(s, z, mask, p)
    w = _dev(single_weight_dict(p), cuda_device)
    md = None if mask is None else mask.to(cuda_device)

    def rank_fn(r, comm):
        sh = S.shard_plan(n, world, r)
        z_loc = S.local_rows(z.to(cuda_device), sh)
        s_buf = S.single_buffer(s.to(cuda_device), sh)
        ph = S.CudaPhases("strict")
        S.sharded_single_block(s_buf, z_loc, md, w, sh, comm, ph)
        torch.cuda.synchronize(cuda_device)
        ph.check()
        return s_buf[:n].cpu()

    for full in run_threads(world, rank_fn):
        assert O.rel_max_err(full, ref) <= O.STRICT_TOL
