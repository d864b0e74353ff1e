"""GPU parity of the fused triangle attention (C-ABI ``fpb_triattn``)
against the CPU oracle (``adapters/atlasfold/runtime.py:32-71`` semantics).

Covers starting / ending node, no mask, random masks with fully masked rows
and columns (uniform weights, no NaN: ``test_triangle_attention.py:54-74``),
padding masks, gate / output biases, and ragged N (not a multiple of the
128-query or 64-key tiles). Tolerances: strict 1e-4, fast 1e-2 of the output
scale.
"""
import pytest
import torch

from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu


def _weights(p, device):
    out = {k: getattr(p, k).to(device) for k in
           ("ln_w", "ln_b", "w_q", "w_k", "w_v", "w_bias", "w_g", "w_o")}
    out["b_g"] = None if p.b_g is None else p.b_g.to(device)
    out["b_o"] = None if p.b_o is None else p.b_o.to(device)
    return out


def _mask(kind, n):
    if kind == "none":
        return None
    if kind == "padding":
        return O.make_padding_mask(n, max(1, n - 7))
    g = torch.Generator().manual_seed(9)
    m = (torch.rand(n, n, generator=g) > 0.3).float()
    m[min(2, n - 1), :] = 0.0
    m[:, min(4, n - 1)] = 0.0
    return m


@pytest.mark.parametrize("n", [7, 33, 96, 124, 144, 200, 257])
@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("precision", ["strict", "fast"])
@pytest.mark.parametrize("mask_kind", ["none", "random", "padding"])
def test_triattn_matches_oracle(cuda_device, n, starting, precision, mask_kind):
    from fireprot_b200 import ops
    z = O.make_pair(n, seed=211 + n)
    p = O.make_triattn_params(seed=3 + int(starting), with_biases=(mask_kind == "random"),
                              ln_affine_random=True)
    mask = _mask(mask_kind, n)
    ref = z + O.triangle_attention(z, mask, p, starting=starting, chunk=32)
    zd = z.to(cuda_device)
    ptr = zd.data_ptr()
    out, ws = ops.triattn(zd, None if mask is None else mask.to(cuda_device),
                          _weights(p, cuda_device), starting=starting, precision=precision,
                          return_workspace=True)
    assert ops.workspace_status(ws) == 0
    assert out.data_ptr() == ptr
    assert torch.isfinite(out).all()
    err = O.rel_max_err(out, ref)
    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
    assert err <= tol, err
    # the update alone must also be accurate (not hidden by the residual)
    err_d = O.rel_max_err(out.cpu() - z, ref - z)
    assert err_d <= (5 * tol), err_d


def test_triattn_c1_known_answer(cuda_device):
    """N=124, seed 0, mask all ones, H=4, d=32."""
    from fireprot_b200 import ops
    n = 124
    z = O.make_pair(n, seed=0)
    p = O.make_triattn_params(seed=1)
    mask = torch.ones(n, n)
    ref = z + O.triangle_attention(z, mask, p, starting=True)
    out = ops.triattn(z.to(cuda_device), mask.to(cuda_device), _weights(p, cuda_device),
                      starting=True, precision="strict")
    assert O.rel_max_err(out, ref) <= O.STRICT_TOL


@pytest.mark.parametrize("n", [48, 96, 100, 144, 300])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_attention_core_key_tile_weights(cuda_device, n, precision):
    """Uniform softmax (q = 0, zero bias) over V that one-hot encodes each
    key's 48-key tile and carries the key index: every output row must give
    each key tile its share of the weight and the mean key index, whatever
    the number of key tiles and whether the last one is full."""
    from fireprot_b200 import ops
    q = torch.zeros(1, 4, n, 32, device=cuda_device)
    k = torch.randn(1, 4, n, 32, generator=torch.Generator().manual_seed(n)).to(cuda_device)
    v = torch.zeros(1, 4, n, 32)
    keys = torch.arange(n)
    v[0, :, keys, torch.clamp(keys // 48, max=30)] = 1.0
    v[0, :, :, 31] = keys.float()
    tb = torch.zeros(1, 4, n, n, device=cuda_device)
    o = ops.attention_core(q, k, v.to(cuda_device), [tb], precision=precision).cpu()
    expect = torch.zeros(32)
    for t in range((n + 47) // 48):
        expect[min(t, 30)] += min(48, n - 48 * t) / n
    expect[31] = (n - 1) / 2
    tol = 1e-5 if precision == "strict" else 1e-2
    for h in range(4):
        err = (o[0, :, h] - expect).abs() / expect.abs().clamp(min=1.0)
        assert err.max().item() <= tol, (h, o[0, 0, h, :8], expect[:8])


@pytest.mark.parametrize("side", ["start", "end"])
def test_fast_mode_against_atlasfold_bf16_storage(cuda_device, side):
    """Fast mode (BF16 operands, FP32 accumulation and softmax) against the
    AtlasFold BF16 path's own output (``adapters/atlasfold/runtime.py:32-71``
    on BF16 modules and z, golden ``triattn_bf16_n64_*``) on the same
    BF16-valued inputs: the result z + update within 1e-2 of the output
    scale; the update alone within 2e-2 of its scale, since the reference's
    BF16 storage itself sits 9.3e-3 from the FP32 math (pinned in
    ``test_oracle_golden.py``) and the fast mode's own error adds to it."""
    from fireprot_b200 import ops
    from tests.test_oracle_golden import bf16_attention_case
    z, mask, p, ref, meta = bf16_attention_case(side)
    delta = torch.empty_like(z).to(cuda_device)
    ops.triattn(z.to(cuda_device), mask.to(cuda_device), _weights(p, cuda_device),
                starting=meta["starting"], precision="fast", delta_out=delta)
    got = delta.cpu()
    assert O.rel_max_err(z + got, z + ref) <= O.FAST_TOL
    assert O.rel_max_err(got, ref) <= 2 * O.FAST_TOL
