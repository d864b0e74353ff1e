"""GPU parity of the channels-last triangle contraction
(``fpb_triangle_contract``, ESMFold2's ``_triangular_contract_chunked``)
against the oracle pinned to the reference's ``packed_contract``: strict
1e-4 / fast 1e-2 of the output scale, both directions, ragged n (vs. the
128-row and 32-key tiles), C = 32 and the ESMFold2 width 256, and the same
call made by a block inside the scope."""
import pytest
import torch
from torch import nn

from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,c", [(1, 32), (7, 32), (33, 64), (130, 256), (257, 32)])
@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_triangle_contract_matches_oracle(cuda_device, n, c, outgoing, precision):
    from fireprot_b200 import ops
    left = O.make_pair(n, c, seed=n + c)
    right = O.make_pair(n, c, seed=n + c + 1)
    ref = O.triangle_contract(left.double(), right.double(), outgoing=outgoing)
    out, ws = ops.triangle_contract(left.to(cuda_device).unsqueeze(0),
                                    right.to(cuda_device).unsqueeze(0), outgoing=outgoing,
                                    precision=precision, return_workspace=True)
    assert ops.workspace_status(ws) == 0
    assert tuple(out.shape) == (1, n, n, c)
    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
    assert O.rel_max_err(out[0], ref) <= tol


class Block(nn.Module):
    def __init__(self, flow):
        super().__init__()
        self.flow = flow
        self.native_calls = 0

    def _triangular_contract_chunked(self, left, right, chunk_size):
        self.native_calls += 1
        return O.triangle_contract(left, right, outgoing=self.flow == "outgoing")


def test_scope_runs_the_b200_contraction(cuda_device):
    from fireprot_b200.esmfold2 import patched_blocks
    m = nn.Module()
    m.folding_trunk = nn.ModuleList([Block("outgoing"), Block("incoming")])
    left = O.make_pair(96, 256, seed=1).unsqueeze(0).to(cuda_device)
    right = O.make_pair(96, 256, seed=2).unsqueeze(0).to(cuda_device)
    with torch.no_grad(), patched_blocks(m, Block) as disp:
        for blk in m.folding_trunk:
            out = blk._triangular_contract_chunked(left, right, 64)
            ref = O.triangle_contract(left.cpu().double(), right.cpu().double(),
                                      outgoing=blk.flow == "outgoing")
            assert O.rel_max_err(out, ref) <= O.STRICT_TOL
            assert blk.native_calls == 0
        # under autograd the block's own method runs
        with torch.enable_grad():
            m.folding_trunk[0]._triangular_contract_chunked(left, right, 64)
        assert m.folding_trunk[0].native_calls == 1
        assert disp.calls == 2
