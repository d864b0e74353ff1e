"""GPU parity of the OpenFold3 ``_attention`` scope on the B200 attention
core. A stand-in module's ``_attention`` is the upstream math (QK^T, add the
biases in order, softmax, PV; ``attention.py:135-148`` runs the same einsums
natively); inside the scope an accepted call must match the float64 oracle
within the strict bound (1e-4 of the output scale; fast mode 1e-2), for
broadcast and per-batch masks, strided views, ragged N and fully masked
rows, and an unaccepted call must reach the stand-in unchanged."""
from types import SimpleNamespace

import pytest
import torch

from oracle import pairformer_oracle as O

pytestmark = pytest.mark.gpu


def upstream_attention(query, key, value, biases, use_high_precision=False):
    a = torch.matmul(query, key.transpose(-1, -2))
    for b in biases:
        a = a + b
    return torch.matmul(torch.softmax(a, dim=-1), value)


def _inputs(b, n, device, *, mask_batch, dead_rows=False, strided=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    if strided:  # [B, N, 4, 32] storage viewed as [B, 4, N, 32]
        q, k, v = (torch.randn(b, n, 4, 32, generator=g).transpose(1, 2) for _ in range(3))
    else:
        q, k, v = (torch.randn(b, 4, n, 32, generator=g) for _ in range(3))
    q = q / 32 ** 0.5
    valid = (torch.rand(mask_batch, n, generator=g) > 0.2).float()
    if dead_rows:
        valid[0] = 0.0  # every key masked for batch entry 0
    mask = (O.MASK_INF * (valid - 1.0)).view(mask_batch, 1, 1, n)
    bias = torch.randn(1, 4, n, n, generator=g)
    if strided:
        bias = bias.transpose(-1, -2).contiguous().transpose(-1, -2)
    to = lambda t: t.to(device)  # noqa: E731
    return to(q), to(k), to(v), [to(mask), to(bias)]


def _oracle(q, k, v, biases, dtype=torch.float64):
    d = [t.detach().cpu().to(dtype) for t in (q, k, v)]
    return O.attention_core(*d, [bb.detach().cpu().to(dtype) for bb in biases])


@pytest.mark.parametrize("n", [7, 33, 200, 1000])
@pytest.mark.parametrize("mask_batch", ["shared", "per_batch"])
@pytest.mark.parametrize("precision", ["strict", "fast"])
def test_scope_runs_the_attention_core(cuda_device, n, mask_batch, precision):
    from fireprot_b200 import backend
    from fireprot_b200.openfold3 import AttentionCoreKernel, AttentionDispatcher, _scoped_hook
    b = 3 if n < 1000 else 1
    q, k, v, biases = _inputs(b, n, cuda_device, mask_batch=1 if mask_batch == "shared" else b,
                              seed=n)
    ref = _oracle(q, k, v, biases)
    mod = SimpleNamespace(_attention=upstream_attention)
    disp = AttentionDispatcher(AttentionCoreKernel(cuda_device.index))
    old = backend.get_precision()
    backend.set_precision(precision)
    try:
        with torch.no_grad(), _scoped_hook(mod, disp):
            out = mod._attention(q, k, v, biases)
    finally:
        backend.set_precision(old)
    assert tuple(out.shape) == (b, 4, n, 32) and out.dtype == torch.float32
    assert disp.kernel.launches_submitted == 1
    tol = O.STRICT_TOL if precision == "strict" else O.FAST_TOL
    assert O.rel_max_err(out, ref) <= tol


def test_strided_views_dead_rows_and_high_precision(cuda_device):
    from fireprot_b200 import backend
    from fireprot_b200.openfold3 import AttentionCoreKernel, AttentionDispatcher, _scoped_hook
    q, k, v, biases = _inputs(2, 150, cuda_device, mask_batch=2, dead_rows=True, strided=True,
                              seed=5)
    # FP32 reference: a fully masked row is a uniform softmax in FP32 (every
    # logit rounds to -1e9), which FP64 does not reproduce
    ref = _oracle(q, k, v, biases, dtype=torch.float32)
    mod = SimpleNamespace(_attention=upstream_attention)
    disp = AttentionDispatcher(AttentionCoreKernel(cuda_device.index))
    old = backend.get_precision()
    backend.set_precision("fast")
    try:
        with torch.no_grad(), _scoped_hook(mod, disp):
            out = mod._attention(q, k, v, biases, use_high_precision=True)  # strict
    finally:
        backend.set_precision(old)
    assert torch.isfinite(out).all()  # dead rows: uniform weights, as in FP32 upstream
    assert O.rel_max_err(out, ref) <= O.STRICT_TOL


@pytest.mark.parametrize("case", ["grad", "one_bias", "cpu"])
def test_unaccepted_calls_reach_upstream(cuda_device, case):
    from fireprot_b200.openfold3 import AttentionCoreKernel, AttentionDispatcher, _scoped_hook
    q, k, v, biases = _inputs(2, 40, cuda_device, mask_batch=2, seed=7)
    if case == "one_bias":
        biases = biases[1:]
    if case == "cpu":
        q, k, v, biases = q.cpu(), k.cpu(), v.cpu(), [bb.cpu() for bb in biases]
    calls = []

    def stand_in(*args, **kwargs):
        calls.append(1)
        return upstream_attention(*args, **kwargs)

    mod = SimpleNamespace(_attention=stand_in)
    disp = AttentionDispatcher(AttentionCoreKernel(cuda_device.index))
    with _scoped_hook(mod, disp):
        if case == "grad":
            with torch.enable_grad():
                mod._attention(q, k, v, biases)
        else:
            with torch.no_grad():
                mod._attention(q, k, v, biases)
    assert calls == [1] and disp.kernel.launches_submitted == 0
