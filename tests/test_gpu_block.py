"""GPU parity of the whole pair stack of one Pairformer block
(``fpb_pair_block``) against the CPU oracle, plus the launch-timing hook."""
import pytest
import torch

from oracle import pairformer_oracle as O
from tests.block_util import block_params

pytestmark = pytest.mark.gpu


def _block(seed):
    from fireprot_b200.modules import PairformerPairBlock
    b = PairformerPairBlock().init_random_(seed)
    g = torch.Generator().manual_seed(seed + 100)
    for m in (b.tri_att_start.mha, b.tri_att_end.mha):
        m.linear_g.bias.data.copy_(torch.randn(128, generator=g))
        m.linear_o.bias.data.copy_(0.1 * torch.randn(128, generator=g))
    for ln in [mod for mod in b.modules() if isinstance(mod, torch.nn.LayerNorm)]:
        ln.weight.data.copy_(1 + 0.1 * torch.randn(ln.weight.shape, generator=g))
        ln.bias.data.copy_(0.1 * torch.randn(ln.bias.shape, generator=g))
    return b


@pytest.mark.parametrize("n", [33, 124])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_pair_block_matches_oracle(cuda_device, n, precision):
    from fireprot_b200 import ops
    b = _block(5)
    ref_p = block_params(b)
    z = O.make_pair(n, seed=77)
    mask = O.make_padding_mask(n, n - 4)
    ref = O.pair_block(z, mask, ref_p, attn_chunk=32)
    bd = b.to(cuda_device)
    zd = z.to(cuda_device)
    out, ws = ops.pair_block(zd, mask.to(cuda_device), bd.c_weights(), precision=precision,
                             return_workspace=True)
    assert ops.workspace_status(ws) == 0
    assert out.data_ptr() == zd.data_ptr()
    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
    # five chained updates: allow the per-op tolerance to accumulate
    assert O.rel_max_err(out, ref) <= 5 * tol


def test_timing_hook_counts_launches(cuda_device):
    from fireprot_b200 import ops
    b = _block(6).to(cuda_device)
    z = O.make_pair(40, seed=1).to(cuda_device)
    ops.timing_enable(True)
    ops.pair_block(z, None, b.c_weights(), precision="strict")
    rec = ops.timing_collect()
    ops.timing_enable(False)
    for k in ("trimul_proj", "contract_strict", "trimul_out", "triattn_proj", "triattn_core",
              "triattn_out", "transition"):
        assert k in rec, rec
    assert rec["triattn_core"]["launches"] == 2
    assert rec["contract_strict"]["launches"] == 2
    assert all(v["total_ms"] > 0 for v in rec.values())
