"""Registry policy contract (CPU): the C++ core behind the reference's
Python API. Mirrors the reference's registry tests
(``tests/operators/test_registry.py``, ``test_rust_registry.py``): priority
order with name tie-break, rejection reasons, failing predicates, per-signature
cache, native fallback counts, manifest shape, escaping interrupts."""
from __future__ import annotations

import json
import os
import sys
import types
from pathlib import Path

import pytest

from fireprot_b200.registry import (OperationRegistry, OperationSignature, PolicyCore,
                                    get_registry, signature_from_tensor)


def _sig(**kw):
    base = dict(operation="op", device_type="cuda", architecture="sm_100", dtype="float32",
                shape=(8, 8, 128))
    base.update(kw)
    return OperationSignature.create(**base)


def test_priority_then_name_order_and_reasons():
    r = OperationRegistry()
    r.register(operation="op", name="zeta", function=lambda: "zeta", supports=lambda s: True,
               priority=5)
    r.register(operation="op", name="alpha", function=lambda: "alpha", supports=lambda s: True,
               priority=5)
    r.register(operation="op", name="high", function=lambda: "high",
               supports=lambda s: (False, "not this one"), priority=9)
    sel = r.resolve(_sig())
    assert sel.implementation.name == "alpha"
    assert sel.rejected == (("high", "not this one"),)
    assert r.dispatch(_sig(), lambda: "native") == "alpha"


def test_failing_predicate_rejects_only_its_candidate():
    r = OperationRegistry()
    r.register(operation="op", name="boom", function=lambda: 1, supports=lambda s: 1 / 0,
               priority=3)
    r.register(operation="op", name="ok", function=lambda: 2, supports=lambda s: True)
    sel = r.resolve(_sig())
    assert sel.implementation.name == "ok"
    assert sel.rejected[0][0] == "boom" and "capability error" in sel.rejected[0][1]


def test_cache_counts_native_and_manifest():
    r = OperationRegistry()
    calls = []

    def sup(s):
        calls.append(s)
        return s.shape[0] == 8

    r.register(operation="op", name="impl", function=lambda: "impl", supports=sup, priority=1)
    assert r.resolve(_sig()).cache_hit is False
    assert r.resolve(_sig()).cache_hit is True
    assert len(calls) == 1
    assert r.dispatch(_sig(shape=(9, 9, 128)), lambda: "native") == "native"
    m = r.manifest()
    counts = {(c["operation"], c["implementation"]): c["count"] for c in m["selection_counts"]}
    assert counts[("op", "impl")] == 2 and counts[("op", "native")] == 1
    assert m["implementations"]["op"] == [{"name": "impl", "priority": 1, "version": "1"}]
    assert {d["selected"] for d in m["decisions"]} == {"impl", "native"}
    assert m["policy_engine"]["name"] == "fireprot-b200-core"
    r.clear_runtime_state()
    assert r.manifest()["selection_counts"] == []
    assert r.resolve(_sig()).cache_hit is False


def test_registration_invalidates_cache_and_errors():
    r = OperationRegistry()
    r.register(operation="op", name="a", function=lambda: "a", supports=lambda s: True)
    r.resolve(_sig())
    r.register(operation="op", name="b", function=lambda: "b", supports=lambda s: True,
               priority=2)
    sel = r.resolve(_sig())
    assert sel.cache_hit is False and sel.implementation.name == "b"
    with pytest.raises(ValueError):
        r.register(operation="op", name="b", function=lambda: 0, supports=lambda s: True)
    with pytest.raises(ValueError):
        r.register(operation="op", name=" ", function=lambda: 0, supports=lambda s: True)
    with pytest.raises(TypeError):
        r.register(operation="op", name="c", function=None, supports=lambda s: True)
    r.unregister("op", "b")
    assert r.resolve(_sig()).implementation.name == "a"
    with pytest.raises(KeyError):
        r.unregister("op", "missing")


def test_keyboard_interrupt_escapes_and_is_not_cached():
    r = OperationRegistry()
    state = {"raise": True}

    def sup(s):
        if state["raise"]:
            raise KeyboardInterrupt
        return True

    r.register(operation="op", name="x", function=lambda: "x", supports=sup)
    with pytest.raises(KeyboardInterrupt):
        r.resolve(_sig())
    assert r.manifest()["selection_counts"] == []
    state["raise"] = False
    sel = r.resolve(_sig())
    assert sel.implementation.name == "x" and sel.cache_hit is False


def test_signature_from_tensor_matches_reference_fields():
    import torch
    t = torch.zeros(4, 4, 128).transpose(0, 1)
    s = signature_from_tensor("op", t, architecture="sm_100", mode="inference", mask="none",
                              inplace=False, attributes={"b": 2, "a": 1})
    assert s.layout == "strided" and s.strides == (128, 512, 1)
    assert s.attributes == (("a", "1"), ("b", "2"))
    assert set(s.as_dict()) == {"operation", "device_type", "architecture", "dtype", "shape",
                                "layout", "mode", "mask", "inplace", "attributes", "strides"}


def test_process_registry_is_shared():
    assert get_registry() is get_registry()


REFERENCE = Path(os.environ.get("FIREPROT_REFERENCE",
                                Path(__file__).resolve().parents[1].parent / "reference")) / "python"


@pytest.mark.skipif(not (REFERENCE / "fireprot/ops/registry.py").exists(),
                    reason="reference checkout not present")
def test_reference_registry_runs_on_this_core(monkeypatch):
    """The reference's own ``fireprot/ops/registry.py`` runs unchanged with
    this C++ core standing in for its Rust bridge."""
    bridge = types.ModuleType("fireprot.ops._bridge")
    bridge.bridge = types.SimpleNamespace(OperatorRegistry=PolicyCore)
    bridge.identity = {"name": "fireprot-b200-core", "bridge_abi": 1}
    saved = {k: v for k, v in sys.modules.items() if k == "fireprot" or k.startswith("fireprot.")}
    for k in saved:
        del sys.modules[k]
    monkeypatch.syspath_prepend(str(REFERENCE))
    sys.modules["fireprot.ops._bridge"] = bridge
    try:
        from fireprot.ops import registry as ref
        r = ref.OperationRegistry()
        r.register(operation="triangle_multiplication", name="b200", function=lambda: "b200",
                   supports=lambda s: (s.architecture == "sm_100", "not sm_100"), priority=50)
        r.register(operation="triangle_multiplication", name="amd", function=lambda: "amd",
                   supports=lambda s: (False, "architecture is not gfx90a"), priority=40)
        sig = ref.OperationSignature.create(operation="triangle_multiplication",
                                            device_type="cuda", architecture="sm_100",
                                            dtype="float32", shape=(4, 4, 128))
        assert r.dispatch(sig, lambda: "native") == "b200"
        other = ref.OperationSignature.create(operation="triangle_multiplication",
                                              device_type="cuda", architecture="gfx90a",
                                              dtype="float32", shape=(4, 4, 128))
        sel = r.resolve(other)
        assert sel.implementation is None
        assert sel.rejected == (("b200", "not sm_100"), ("amd", "architecture is not gfx90a"))
        m = r.manifest()
        assert m["policy_engine"]["name"] == "fireprot-b200-core"
        assert {c["implementation"] for c in m["selection_counts"]} == {"b200", "native"}
        json.dumps(m)
    finally:
        for k in [k for k in sys.modules if k == "fireprot" or k.startswith("fireprot.")]:
            del sys.modules[k]
        sys.modules.update(saved)
