"""GPU parity of the fused pair transition (C-ABI ``fpb_transition``) against
the CPU oracle (``recycle.py:203-227`` semantics), strict 1e-4 / fast 1e-2."""
import pytest
import torch

from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 7, 33, 124, 200])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_transition_matches_oracle(cuda_device, n, precision):
    from fireprot_b200 import ops
    z = O.make_pair(n, seed=401 + n)
    p = O.make_transition_params(seed=11, ln_affine_random=True)
    ref = z + O.pair_transition(z, p)
    zd = z.to(cuda_device)
    w = {k: getattr(p, k).to(cuda_device) for k in ("ln_w", "ln_b", "w_a", "w_b", "w_out")}
    out, ws = ops.transition(zd, w, precision=precision, return_workspace=True)
    assert ops.workspace_status(ws) == 0
    assert out.data_ptr() == zd.data_ptr()
    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
    assert O.rel_max_err(out, ref) <= tol
    assert O.rel_max_err(out.cpu() - z, ref - z) <= 5 * tol


def test_transition_large_means_and_constant_rows(cuda_device):
    """LN robustness as in test_packed_triangle.py:71-83: +1000 offsets and a
    constant row (variance 0) stay finite and accurate."""
    from fireprot_b200 import ops
    z = O.make_pair(9, seed=5) + 1000.0
    z[0, 0] = 1000.0
    p = O.make_transition_params(seed=12)
    ref = z.double() + O.pair_transition(z.double(), O.TransitionParams(
        *(t.double() for t in (p.ln_w, p.ln_b, p.w_a, p.w_b, p.w_out))))
    w = {k: getattr(p, k).to(cuda_device) for k in ("ln_w", "ln_b", "w_a", "w_b", "w_out")}
    out = ops.transition(z.to(cuda_device), w, precision="strict")
    assert torch.isfinite(out).all()
    assert O.rel_max_err(out.cpu() - z, (ref - z.double()).float()) <= 1e-3
