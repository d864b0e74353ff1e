"""GPU tests of the drop-in dispatch boundary (``fireprot_b200.backend``)
with Protenix-shaped modules, against the CPU oracle. Each call must select
the b200 implementation (registry manifest) and match the oracle within the
precision's tolerance; inputs stay unmodified where the reference contract
says so (``test_ck_attention.py:81``)."""
import math

import pytest
import torch

from oracle import pairformer_oracle as O
from tests.block_util import transition_params, triattn_params, trimul_params

pytestmark = pytest.mark.gpu


def _block(dev, seed=21):
    from fireprot_b200.modules import PairformerPairBlock
    b = PairformerPairBlock().init_random_(seed)
    g = torch.Generator().manual_seed(seed)
    for m in (b.tri_att_start.mha, b.tri_att_end.mha):
        m.linear_g.bias.data.copy_(torch.randn(128, generator=g))
        m.linear_o.bias.data.copy_(0.1 * torch.randn(128, generator=g))
    return b.to(dev).eval()


def _selected(op):
    from fireprot_b200 import backend
    m = backend.get_registry().manifest()
    return {c["implementation"] for c in m["selection_counts"] if c["operation"] == op}


@pytest.mark.parametrize("precision", ["strict", "fast"])
@pytest.mark.parametrize("outgoing", [True, False])
def test_dispatch_triangle_multiplication(cuda_device, precision, outgoing):
    from fireprot_b200 import backend
    backend.set_precision(precision)
    try:
        blk = _block(cuda_device)
        mod = blk.tri_mul_out if outgoing else blk.tri_mul_in
        n = 77
        z = O.make_pair(n, seed=5)
        mask = O.make_padding_mask(n, 70)
        ref = O.triangle_multiplication(z, mask, trimul_params(mod), outgoing=outgoing, add=True)
        zd = z.to(cuda_device)
        with torch.no_grad():
            out = backend.dispatch_triangle_multiplication(
                module=mod, z=zd, mask=mask.to(cuda_device), inplace_safe=True,
                add_with_inplace=True, inplace_chunk_size=256,
                native=lambda **_: pytest.fail("native path taken"))
        assert out.data_ptr() == zd.data_ptr()
        tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
        assert O.rel_max_err(out, ref) <= tol
        assert backend.TRIMUL_IMPL in _selected(backend.TRIMUL)
    finally:
        backend.set_precision("strict")


@pytest.mark.parametrize("with_mask", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_dispatch_triangle_attention_core(cuda_device, with_mask, precision):
    """q/k/v in Protenix's head-major strided views, non-contiguous triangle
    bias (heads fastest), [B,1,1,N] mask bias incl. a dead row."""
    from fireprot_b200 import backend
    backend.set_precision(precision)
    try:
        b, n = 19, 67
        g = torch.Generator().manual_seed(521)
        x = torch.randn(b, n, 3 * 128, generator=g)
        q, k, v = (t.reshape(b, n, 4, 32).transpose(1, 2) for t in x.split(128, dim=-1))
        q = q / math.sqrt(32)
        tri = torch.randn(n, n, 4, generator=g).permute(2, 0, 1).unsqueeze(0)
        biases = [tri]
        if with_mask:
            mask = (torch.rand(b, n, generator=g) > 0.2).float()
            mask[3] = 0.0
            biases = [(1e9 * (mask - 1))[:, None, None, :], tri]
        ref = O.attention_core(q, k, v, biases).transpose(-2, -3)
        dev_b = [t.to(cuda_device) for t in biases]
        xd = x.to(cuda_device)
        qd, kd, vd = (t.reshape(b, n, 4, 32).transpose(1, 2) for t in xd.split(128, dim=-1))
        qd = qd / math.sqrt(32)
        before = xd.clone()
        with torch.no_grad():
            out = backend.dispatch_triangle_attention(
                module=None, q=qd, k=kd, v=vd, biases=dev_b,
                native=lambda **_: pytest.fail("native path taken"))
        assert tuple(out.shape) == (b, n, 4, 32)
        assert torch.equal(xd, before)
        assert torch.isfinite(out).all()
        tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
        assert O.rel_max_err(out, ref) <= tol
        assert backend.TRIATT_IMPL in _selected(backend.TRIATT)
    finally:
        backend.set_precision("strict")


@pytest.mark.parametrize("starting", [True, False])
def test_triangle_attention_module_returns_delta(cuda_device, starting):
    from fireprot_b200 import backend
    blk = _block(cuda_device)
    mod = blk.tri_att_start if starting else blk.tri_att_end
    n = 45
    z = O.make_pair(n, seed=8)
    mask = O.make_padding_mask(n, 40)
    ref = O.triangle_attention(z, mask, triattn_params(mod), starting=starting)
    zd = z.to(cuda_device)
    before = zd.clone()
    with torch.no_grad():
        delta = backend.triangle_attention_module(
            module=mod, z=zd, mask=mask.to(cuda_device), starting=starting,
            native=lambda **_: pytest.fail("native path taken"))
    assert torch.equal(zd, before)
    assert O.rel_max_err(delta, ref) <= O.STRICT_TOL


def test_dispatch_transition_returns_delta(cuda_device):
    from fireprot_b200 import backend
    blk = _block(cuda_device)
    z = O.make_pair(33, seed=2)
    ref = O.pair_transition(z, transition_params(blk.pair_transition))
    zd = z.to(cuda_device)
    before = zd.clone()
    with torch.no_grad():
        delta = backend.dispatch_transition(module=blk.pair_transition, x=zd,
                                            native=lambda: pytest.fail("native path taken"))
    assert torch.equal(zd, before)
    assert O.rel_max_err(delta, ref) <= O.STRICT_TOL


def test_training_mode_goes_native(cuda_device):
    from fireprot_b200 import backend
    blk = _block(cuda_device)
    z = torch.randn(8, 8, 128, device=cuda_device)
    with torch.enable_grad():
        r = backend.dispatch_transition(module=blk.pair_transition, x=z, native=lambda: "native")
    assert r == "native"
