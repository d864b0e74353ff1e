"""CPU checks of the ESMFold2 triangle-contraction scope: blocks outside the
scoped sub-trees are left alone, a second replacement is refused, the
original methods come back on exit (and a foreign replacement is detected),
calls the B200 kernel does not take (CPU tensors here) run the block's own
method with its own arguments, and the oracle matches a chunked
restatement of the native loop."""
import pytest
import torch
from torch import nn

from fireprot_b200.esmfold2 import METHOD, patched_blocks
from oracle import pairformer_oracle as O


class Block(nn.Module):
    def __init__(self, flow):
        super().__init__()
        self.flow = flow
        self.seen = []

    def _triangular_contract_chunked(self, left, right, chunk_size):
        self.seen.append(chunk_size)
        return O.triangle_contract(left, right, outgoing=self.flow == "outgoing")


class Model(nn.Module):
    def __init__(self):
        super().__init__()
        self.folding_trunk = nn.ModuleList([Block("outgoing"), Block("incoming")])
        self.diffusion = nn.ModuleList([Block("outgoing")])


def test_scope_patches_only_the_listed_subtrees_and_restores():
    m = Model()
    with torch.no_grad(), patched_blocks(m, Block) as disp:
        assert METHOD in m.folding_trunk[0].__dict__ and METHOD in m.folding_trunk[1].__dict__
        assert METHOD not in m.diffusion[0].__dict__
        x = torch.randn(1, 5, 5, 32)
        for blk in m.folding_trunk:
            out = getattr(blk, METHOD)(x, x, 2)
            ref = O.triangle_contract(x, x, outgoing=blk.flow == "outgoing")
            assert torch.equal(out, ref) and blk.seen == [2]  # CPU: the block's own method
        assert disp.calls == 0
        assert all(d["selected"] == "native" for d in disp.manifest()["registry"]["decisions"])
    assert all(METHOD not in b.__dict__ for b in m.modules() if isinstance(b, Block))


def test_second_scope_and_foreign_replacement_refused():
    m = Model()
    with patched_blocks(m, Block):
        with pytest.raises(RuntimeError, match="already replaced"):
            with patched_blocks(m, Block):
                pass
    with pytest.raises(RuntimeError, match="changed during"):
        with patched_blocks(m, Block):
            setattr(m.folding_trunk[0], METHOD, lambda *a: None)


def test_no_compatible_blocks_is_an_error():
    with pytest.raises(RuntimeError, match="No compatible"):
        with patched_blocks(nn.Linear(2, 2), Block):
            pass


@pytest.mark.parametrize("outgoing", [True, False])
def test_oracle_equals_the_chunked_loop(outgoing):
    """The native loop contracts chunks of i; chunking does not change a
    single output element."""
    g = torch.Generator().manual_seed(3)
    left = torch.randn(1, 11, 11, 32, generator=g, dtype=torch.float64)
    right = torch.randn(1, 11, 11, 32, generator=g, dtype=torch.float64)
    ref = O.triangle_contract(left, right, outgoing=outgoing)
    parts = []
    for s in range(0, 11, 4):
        sl = left[:, s:s + 4] if outgoing else left[:, :, s:s + 4]
        if outgoing:
            parts.append(torch.einsum("bikc,bjkc->bijc", sl, right))
        else:
            parts.append(torch.einsum("bkic,bkjc->bijc", sl, right))
    torch.testing.assert_close(torch.cat(parts, dim=1), ref, rtol=1e-12, atol=1e-12)
