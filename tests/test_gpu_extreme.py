"""The reference's extreme-value attention cases on the B200 attention core.

- A -inf triangle-bias row and a +80 entry at N=1000, through the Protenix
  dispatch (``dispatch_triangle_attention``), inputs left bit-unchanged and a
  contiguous result: ``tests/operators/test_ck_attention.py:56-85`` compares
  its kernel with torch's ``scaled_dot_product_attention`` there, which gives
  0 for a row whose every logit is -inf.
- Every key masked (-1e9) under a linspace(-80, 80) triangle bias:
  ``tests/operators/test_triangle_attention.py:54-74`` (finite, equal to the
  upstream math in FP32).
- The OpenFold3 mask + bias softmax contract that a zero row sum is NaN
  (``kernels/amd/fireprot_softmax_fp32.cpp:61-62``), through the OpenFold3
  scope: a batch entry whose mask is -inf everywhere and a -inf bias row give
  NaN rows there and the upstream result elsewhere.

Tolerances: strict 1e-4, fast 1e-2 of the output scale (finite entries).
"""
from types import SimpleNamespace

import pytest
import torch

from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu


def _tol(precision):
    return O.STRICT_TOL if precision == "strict" else O.FAST_TOL


def _native_fail(**_):
    raise AssertionError("native path selected")


@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_protenix_dispatch_inf_row_and_plus80_n1000(cuda_device, precision):
    from fireprot_b200 import backend
    n = 1000
    g = torch.Generator().manual_seed(521)
    q, k, v = (torch.randn(n, n, 4, 32, generator=g).to(cuda_device).transpose(1, 2)
               for _ in range(3))
    q /= 32 ** 0.5
    saved = [t.clone() for t in (q, k, v)]
    bias = torch.randn(n, n, 4, generator=g).to(cuda_device).permute(2, 0, 1).unsqueeze(0)
    bias_saved = bias.clone()
    batches = [0, 1, 499, 998, 999]
    old = backend.get_precision()
    backend.set_precision(precision)
    try:
        for exceptional in (False, True):
            if exceptional:
                bias[:, :, 0, :] = float("-inf")
                bias[:, :, 1, 0] = 80.0
                bias_saved = bias.clone()
            with torch.no_grad():
                out = backend.dispatch_triangle_attention(
                    module=SimpleNamespace(training=False), q=q, k=k, v=v, biases=[bias],
                    native=_native_fail)
            assert out.is_contiguous() and tuple(out.shape) == (n, n, 4, 32)
            qc, kc, vc = (t[batches].cpu().double() for t in (q, k, v))
            ref = O.attention_core(qc, kc, vc, [bias.cpu().double()], empty_rows="zero")
            ref = ref.transpose(-2, -3)  # [b, N, H, D]
            got = out[batches].cpu()
            if exceptional:
                assert (got[:, 0] == 0).all()  # every logit -inf: 0, as SDPA
                # +80 on key 0 of query 1: the softmax is one-hot on key 0
                # (fast mode reads V in BF16)
                assert torch.allclose(got[:, 1], vc.transpose(1, 2)[:, 0].float(),
                                      atol=1e-4 if precision == "strict" else 3e-2)
            assert torch.isfinite(got).all()
            assert O.rel_max_err(got, ref) <= _tol(precision)
            for t, before in zip((q, k, v, bias), (*saved, bias_saved)):
                assert torch.equal(t, before)
    finally:
        backend.set_precision(old)


@pytest.mark.parametrize("n", [7, 100, 257])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_all_keys_masked_under_linspace_bias(cuda_device, n, precision):
    from fireprot_b200 import ops
    g = torch.Generator().manual_seed(202)
    q, k, v = (torch.randn(5, 4, n, 32, generator=g) for _ in range(3))
    q = q / 32 ** 0.5
    mask_bias = torch.full((5, 1, 1, n), -1e9)
    tri = torch.linspace(-80, 80, n).view(1, 1, 1, n).expand(1, 4, n, n)
    ref = O.attention_core(q, k, v, [mask_bias, tri])  # FP32, the reference's order
    out = ops.attention_core(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                             [mask_bias.to(cuda_device), tri.to(cuda_device)],
                             precision=precision).cpu()
    assert torch.isfinite(out).all()
    assert O.rel_max_err(out, ref.transpose(-2, -3)) <= _tol(precision)


def _upstream_attention(query, key, value, biases, use_high_precision=False):
    a = torch.matmul(query, key.transpose(-1, -2))
    for b in biases:
        a = a + b
    return torch.matmul(torch.softmax(a, dim=-1), value)


@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_openfold3_zero_row_sum_is_nan(cuda_device, precision):
    from fireprot_b200 import backend
    from fireprot_b200.openfold3 import AttentionCoreKernel, AttentionDispatcher, _scoped_hook
    b, n = 3, 150
    g = torch.Generator().manual_seed(613)
    q, k, v = (torch.randn(b, 4, n, 32, generator=g) for _ in range(3))
    q = q / 32 ** 0.5
    valid = (torch.rand(b, n, generator=g) > 0.2).float()
    mask = (O.MASK_INF * (valid - 1.0)).view(b, 1, 1, n)
    mask[1] = float("-inf")               # batch entry 1: no finite logit anywhere
    bias = torch.randn(1, 4, n, n, generator=g)
    bias[0, 2, 5, :] = float("-inf")      # head 2, query 5: no finite logit
    bias[0, 0, 7, :60] = float("-inf")    # partly -inf rows stay finite
    ref = _upstream_attention(q.double(), k.double(), v.double(),
                              [mask.double(), bias.double()])
    dev = [t.to(cuda_device) for t in (q, k, v, mask, bias)]
    mod = SimpleNamespace(_attention=_upstream_attention)
    disp = AttentionDispatcher(AttentionCoreKernel(cuda_device.index))
    old = backend.get_precision()
    backend.set_precision(precision)
    try:
        with torch.no_grad(), _scoped_hook(mod, disp):
            out = mod._attention(dev[0], dev[1], dev[2], [dev[3], dev[4]]).cpu()
    finally:
        backend.set_precision(old)
    assert disp.kernel.launches_submitted == 1
    nan_ref = torch.isnan(ref)
    assert nan_ref[1].all() and nan_ref[:, 2, 5].all()
    assert torch.equal(torch.isnan(out), nan_ref)
    fin = ~nan_ref
    err = (out.double()[fin] - ref[fin]).abs().max() / ref[fin].abs().max()
    assert err.item() <= _tol(precision)
