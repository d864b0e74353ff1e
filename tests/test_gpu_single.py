"""GPU parity of the single stack (C-ABI ``fpb_single_block``) against the
CPU oracle (AlphaFold 3 Algorithms 24 and 11; parity unpinned).

The kernels compute in FP32 on CUDA cores in both precision modes, so both
are held to the strict bound: 1e-4 of the output scale against the FP32
oracle, and against the FP64 oracle on rows with at least one valid key
(fully masked rows are uniform softmaxes in FP32 arithmetic, as in the
reference's FP32 math, and FP64 does not reproduce that rounding)."""
import pytest
import torch

from oracle import pairformer_oracle as O

from sharded_util import oracle_single_params, single_weight_dict

pytestmark = pytest.mark.gpu

TOL = O.STRICT_TOL


def _mask(n, kind):
    if kind == "none":
        return None
    if kind == "padding":
        return O.make_padding_mask(n, max(1, n - 7))
    g = torch.Generator().manual_seed(n)
    return (torch.rand(n, n, generator=g) > 0.25).float()


def _struct(p, device):
    from fireprot_b200 import modules
    keep = []
    w = modules.SingleBlockWeights()
    modules._fill(w, {k: v.to(device) for k, v in single_weight_dict(p).items()}, keep)
    return w, keep


def _valid_rows(mask, n):
    if mask is None:
        return torch.ones(n, dtype=torch.bool)
    return mask.sum(1) > 0


@pytest.mark.parametrize("n", [1, 7, 33, 100, 129, 257])
@pytest.mark.parametrize("mask_kind", ["none", "padding", "random"])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_single_block_matches_oracle(cuda_device, n, mask_kind, precision):
    from fireprot_b200 import ops
    s = O.make_single(n, seed=500 + n)
    z = O.make_pair(n, seed=600 + n)
    mask = _mask(n, mask_kind)
    p = O.make_single_params(seed=17, ln_affine_random=True)
    ref32 = O.single_block(s, z, mask, p)
    p64 = O.make_single_params(seed=17, ln_affine_random=True, dtype=torch.float64)
    ref64 = O.single_block(s.double(), z.double(), None if mask is None else mask.double(), p64)
    w, keep = _struct(p, cuda_device)
    sd = s.to(cuda_device)
    md = None if mask is None else mask.to(cuda_device)
    out, ws = ops.single_block(sd, z.to(cuda_device), md, w, precision=precision,
                               return_workspace=True)
    torch.cuda.synchronize(cuda_device)
    assert ops.workspace_status(ws) == 0
    assert out.data_ptr() == sd.data_ptr()
    out = out.cpu()
    assert torch.isfinite(out).all()
    assert O.rel_max_err(out, ref32) <= TOL
    rows = _valid_rows(mask, n)
    assert O.rel_max_err(out[rows], ref64[rows]) <= TOL
    # the update itself, not only s + update
    assert O.rel_max_err(out - s, ref32 - s) <= 5 * TOL


@pytest.mark.parametrize("n,r0,rows", [(100, 0, 37), (100, 40, 37), (100, 96, 4), (129, 1, 128)])
def test_single_block_row_range(cuda_device, n, r0, rows):
    """A call on query rows [r0, r0 + rows) with those pair rows updates
    exactly those rows of s (every row of s feeds keys and values)."""
    from fireprot_b200 import ops
    s = O.make_single(n, seed=n + r0)
    z = O.make_pair(n, seed=n + rows)
    mask = _mask(n, "random")
    p = O.make_single_params(seed=19, ln_affine_random=True)
    ref = O.single_block(s, z, mask, p)
    w, keep = _struct(p, cuda_device)
    sd = s.to(cuda_device)
    z_loc = z[r0:r0 + rows].contiguous().to(cuda_device)
    ops.single_block(sd, z_loc, mask.to(cuda_device), w, r0=r0)
    out = sd.cpu()
    assert O.rel_max_err(out[r0:r0 + rows], ref[r0:r0 + rows]) <= TOL
    assert torch.equal(out[:r0], s[:r0])
    assert torch.equal(out[r0 + rows:], s[r0 + rows:])


def test_single_module_and_full_block(cuda_device):
    """``PairformerBlock``: pair stack, then the single stack on the updated z."""
    from fireprot_b200 import modules
    from block_util import block_params
    n = 72
    blk = modules.PairformerBlock().init_random_(seed=3).to(cuda_device)
    s = O.make_single(n, seed=1)
    z = O.make_pair(n, seed=2)
    mask = O.make_padding_mask(n, 65)
    pp = block_params(blk.pair)
    z_ref = O.pair_block(z, mask, pp)
    ps = oracle_single_params(blk.single.weight_dict(), dtype=torch.float32)
    s_ref = O.single_block(s, z_ref, mask, ps)
    sd, zd = s.to(cuda_device), z.to(cuda_device)
    blk(sd, zd, mask.to(cuda_device), precision="strict")
    assert O.rel_max_err(zd.cpu(), z_ref) <= TOL
    assert O.rel_max_err(sd.cpu(), s_ref) <= TOL
