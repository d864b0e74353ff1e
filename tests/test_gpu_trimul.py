"""GPU parity of the fused triangle multiplicative update (C-ABI
``fpb_trimul``) against the CPU oracle (Protenix semantics,
``triangle_multiplication.py:162-193``).

Tolerances (north star, relative to the fp32 output scale): strict 1e-4,
fast 1e-2. Cases cover both directions, add / overwrite, no mask, a dense
random mask and a padding mask, ragged sizes (N not a tile multiple) and the
in-place contract (same storage returned, ``test_packed_triangle.py:105``).
"""
import pytest
import torch

from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu


def _weights(p, device):
    return {k: getattr(p, k).to(device) for k in
            ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p", "w_b_g", "w_g", "ln_out_w",
             "ln_out_b", "w_z")}


@pytest.mark.parametrize("n", [7, 33, 124, 200])
@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
@pytest.mark.parametrize("mask_kind", ["none", "random", "padding"])
def test_trimul_matches_oracle(cuda_device, n, outgoing, precision, mask_kind):
    from fireprot_b200 import ops
    z = O.make_pair(n, seed=101 + n)
    p = O.make_trimul_params(seed=7 + int(outgoing), ln_affine_random=True)
    if mask_kind == "none":
        mask = None
    elif mask_kind == "random":
        g = torch.Generator().manual_seed(5)
        mask = (torch.rand(n, n, generator=g) > 0.25).float()
    else:
        mask = O.make_padding_mask(n, max(1, n - 5))
    for add in (True, False):
        ref = O.triangle_multiplication(z, mask, p, outgoing=outgoing, add=add)
        zd = z.to(cuda_device)
        ptr = zd.data_ptr()
        out, ws = ops.trimul(zd, None if mask is None else mask.to(cuda_device),
                             _weights(p, cuda_device), outgoing=outgoing, add=add,
                             precision=precision, return_workspace=True)
        assert ops.workspace_status(ws) == 0
        assert out.data_ptr() == ptr
        err = O.rel_max_err(out, ref)
        tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
        assert err <= tol, (add, err)


def test_trimul_rejects_cpu_and_bad_shapes(cuda_device):
    from fireprot_b200 import ops
    p = O.make_trimul_params()
    with pytest.raises(RuntimeError):
        ops.trimul(torch.randn(8, 8, 128), None, _weights(p, "cpu"), outgoing=True)
    with pytest.raises(RuntimeError):
        ops.trimul(torch.randn(8, 8, 64, device=cuda_device), None, _weights(p, cuda_device),
                   outgoing=True)
