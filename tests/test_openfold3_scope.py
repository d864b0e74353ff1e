"""CPU checks of the OpenFold3 ``_attention`` scope (the reference's
``adapters/openfold3/attention.py:43-148`` interface, exercised the way
``tests/operators/test_openfold3_attention_scope.py`` does): per-context
installation, refusal of a second scope, cleanup on errors and detection of
a foreign replacement, native fallback through the registry with the call's
own arguments, and the tensor contract of accepted calls."""
from concurrent.futures import ThreadPoolExecutor
from contextvars import copy_context
from types import SimpleNamespace

import pytest
import torch

from fireprot_b200.openfold3 import AttentionDispatcher, _scoped_hook, contract_ok


def test_only_the_scoped_context_sees_the_dispatcher():
    def native(x):
        return "native", x

    mod = SimpleNamespace(_attention=native)
    with ThreadPoolExecutor(max_workers=1) as pool:
        with _scoped_hook(mod, lambda original, x: ("scoped", x)):
            assert mod._attention(1) == ("scoped", 1)
            assert pool.submit(mod._attention, 2).result() == ("native", 2)
            kept = mod._attention
            ctx = copy_context()
        assert mod._attention is native
        # a reference kept from inside the scope falls back once it closed
        assert kept(3) == ("native", 3)
        assert ctx.run(kept, 4) == ("native", 4)


def test_second_scope_refused_and_outer_kept():
    mod = SimpleNamespace(_attention=lambda: "native")

    def open_inner():
        with _scoped_hook(mod, lambda original: "inner"):
            pytest.fail("a second scope was installed")

    with _scoped_hook(mod, lambda original: "outer"):
        with pytest.raises(RuntimeError, match="already installed"):
            open_inner()
        with ThreadPoolExecutor(max_workers=1) as pool:
            with pytest.raises(RuntimeError, match="already installed"):
                pool.submit(open_inner).result()
        assert mod._attention() == "outer"
    assert mod._attention() == "native"


def test_errors_restore_and_foreign_replacement_is_left_in_place():
    native = lambda: "native"  # noqa: E731
    mod = SimpleNamespace(_attention=native)
    with pytest.raises(KeyError):
        with _scoped_hook(mod, lambda original: "scoped"):
            raise KeyError("model failure")
    assert mod._attention is native
    foreign = lambda: "foreign"  # noqa: E731
    with pytest.raises(RuntimeError, match="changed during"):
        with _scoped_hook(mod, lambda original: "scoped"):
            mod._attention = foreign
    assert mod._attention is foreign
    # the guard was released: a new scope works over the foreign function
    with _scoped_hook(mod, lambda original: original()):
        assert mod._attention() == "foreign"


def test_native_fallback_keeps_the_call_arguments():
    disp = AttentionDispatcher(None)
    q = torch.zeros(1, 4, 3, 32)
    biases = [torch.zeros(1)]
    seen = []

    def native(qq, kk, vv, bb, use_high_precision=False):
        seen.append((qq, kk, vv, bb, use_high_precision))
        return qq

    with torch.no_grad():
        for _ in range(2):
            assert disp(native, q, q, q, biases, True) is q
    assert len(seen) == 2
    assert all(c[3] is biases and c[4] is True for c in seen)
    report = disp.manifest()
    assert report["kernel"] is None and report["launches_submitted"] == 0
    assert all(d["selected"] == "native" for d in report["registry"]["decisions"])


def _case(b=2, n=9, mask_batch=None):
    q = torch.randn(b, 4, n, 32)
    mask = torch.zeros(b if mask_batch is None else mask_batch, 1, 1, n)
    bias = torch.randn(1, 4, n, n)
    return q, q.clone(), q.clone(), [mask, bias]


def test_contract_accepts_the_attention_core_shapes():
    q, k, v, biases = _case()
    assert contract_ok(q, k, v, biases)
    assert contract_ok(q, k, v, [biases[0][:1], biases[1]])           # mask shared by the batch
    qt = torch.randn(2, 9, 4, 32).transpose(1, 2)                       # strided q
    assert contract_ok(qt, k, v, [biases[0], biases[1].transpose(-1, -2)])
    assert contract_ok(*_case(b=1, n=1))


@pytest.mark.parametrize("case", ["one_bias", "three_biases", "heads", "dim", "mask_shape",
                                  "bias_shape", "dtype", "grad", "kv_shape", "not_tensor"])
def test_contract_rejects(case):
    q, k, v, biases = _case()
    if case == "one_bias":
        biases = biases[1:]
    elif case == "three_biases":
        biases = biases + [biases[1]]
    elif case == "heads":
        q = k = v = torch.randn(2, 8, 9, 32)
    elif case == "dim":
        q = k = v = torch.randn(2, 4, 9, 16)
    elif case == "mask_shape":
        biases = [torch.zeros(2, 1, 9, 9), biases[1]]
    elif case == "bias_shape":
        biases = [biases[0], torch.zeros(2, 4, 9, 9)]
    elif case == "dtype":
        q = q.double()
    elif case == "grad":
        q = q.clone().requires_grad_()
    elif case == "kv_shape":
        k = torch.randn(2, 4, 8, 32)
    elif case == "not_tensor":
        biases = [biases[0], 0.0]
    assert not contract_ok(q, k, v, biases)
