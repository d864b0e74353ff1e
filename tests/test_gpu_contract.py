"""GPU parity of the tcgen05 batched triangle contraction (C-ABI
``fpb_packed_bmm``) against the float64 product of the same inputs.

Strict (3xTF32) must stay within 1e-4 of the output scale and fast (BF16)
within 1e-2; both directions of ``lt_bmm.packed_bmm`` (``lt_bmm.py:85``).
"""
import pytest
import torch

from oracle.pairformer_oracle import FAST_TOL, STRICT_TOL, rel_max_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [7, 33, 124, 257, 512])
@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_packed_bmm_matches_float64(cuda_device, n, outgoing, precision):
    from fireprot_b200 import ops
    g = torch.Generator().manual_seed(317 + n)
    batch = 3
    a = torch.randn(batch, n, n, generator=g)
    b = torch.randn(batch, n, n, generator=g)
    ref = a.double() @ b.double().transpose(-1, -2) if outgoing else \
        a.double().transpose(-1, -2) @ b.double()
    out, ws = ops.packed_bmm(a.to(cuda_device), b.to(cuda_device), outgoing, precision,
                             return_workspace=True)
    assert ops.workspace_status(ws) == 0
    err = rel_max_err(out, ref)
    tol = STRICT_TOL if precision == "strict" else FAST_TOL
    assert err <= tol, err
    if precision == "strict":
        # 3xTF32 should be close to fp32 accuracy, far inside the tolerance
        assert err <= 1e-5, err
