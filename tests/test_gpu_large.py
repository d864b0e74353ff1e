"""Full-size parity at the configurations that are timed (GPU).

BASELINE config 2 (one whole block at N=1000, full mask), the headline shape
of config 3 (N=1536, padding mask valid 1480) and config 5 (one strict block
at N=3072, full mask): the block runs one operator at a time on the GPU
(``PairformerBlock.forward_by_operator``, the same kernels as the fused
block), and after every operator 16+ lines of its result (rows; columns for
the ending node) are recomputed by the oracle from the GPU's own input to
that operator (``oracle.block_check``). Every operator of the chain is held
to the north-star bound: strict 1e-4, fast 1e-2 of the output scale (the
update alone to 5x that, as in the per-operator tests). The lines include
the first and last, and around the padding edge. The fused ``fpb_pair_block``
on the same input is checked to give the same pair tensor as the chain.
"""
import pytest
import torch

from oracle import block_check as BC
from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu

CASES = {
    "c2_n1000_full": (1000, None, ("strict", "fast")),
    "c3_n1536_valid1480": (1536, 1480, ("strict", "fast")),
    "c5_n3072_full": (3072, None, ("strict",)),
}


def _params(block):
    pair = {name: getattr(block.pair, name).weight_dict() for name in BC.PAIR_OPERATORS}
    return BC.params_from_weights(pair, block.single.weight_dict())


def _run(cuda_device, n, valid, precision):
    from fireprot_b200.modules import PairformerBlock
    torch.set_num_threads(max(1, torch.get_num_threads()))
    block = PairformerBlock().init_random_(seed=21)
    p, ps = _params(block)
    z = O.make_pair(n, seed=0)
    s = O.make_single(n, seed=1)
    mask = torch.ones(n, n) if valid is None else O.make_padding_mask(n, valid)
    lines = O.sample_lines(n, count=12, seed=n, valid=valid)
    bd = block.to(cuda_device)
    zd, sd, md = z.to(cuda_device), s.to(cuda_device), mask.to(cuda_device)
    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
    errs = {}
    z_in = z
    for name, t in bd.forward_by_operator(sd, zd, md, precision=precision):
        if name == "single":
            errs[name] = BC.check_single(s, t.cpu(), z_in, mask, ps, lines)
            continue
        z_out = t.cpu()
        errs[name] = BC.check_pair_operator(name, z_in, z_out, mask, p, lines)
        z_in = z_out
    assert torch.isfinite(z_in).all()
    for name, e in errs.items():
        assert e["out"] <= tol and e["update"] <= 5 * tol, (name, e)
    # the fused block runs the same kernels in the same order
    zf = z.to(cuda_device)
    bd.pair(zf, md, precision=precision)
    assert O.rel_max_err(zf, z_in) <= 1e-6
    return errs


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_block_operators_at_full_size(cuda_device, case, precision):
    n, valid, precisions = CASES[case]
    if precision not in precisions:
        pytest.skip(f"{case} is a {'/'.join(precisions)} configuration")
    errs = _run(cuda_device, n, valid, precision)
    print(case, precision, {k: {kk: f"{vv:.2e}" for kk, vv in v.items()}
                            for k, v in errs.items()})
