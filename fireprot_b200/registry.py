"""Operator registry with the reference's Python API, on the C++ policy core.

Same surface as ``python/fireprot/ops/registry.py`` (``OperationSignature``
fields and ``create``/``as_dict``, ``OperationRegistry.register / unregister
/ resolve / dispatch / manifest / clear_runtime_state``, the module-level
``registry`` and ``signature_from_tensor``). The policy (priority / name /
version ordering, first passing capability wins, per-signature cache,
selection counts including ``native``, last decisions) lives in the C++ core
of ``libfireprot_b200.so`` (``csrc/registry.cpp``), the counterpart of the
reference's Rust ``crates/fireprot-core/src/registry.rs``. A missing match
always means the caller's native fallback (``registry.py:151-164``).
"""
from __future__ import annotations

import ctypes
import dataclasses
import json
import threading
from collections.abc import Callable, Mapping
from typing import Any

from . import _lib

Capability = Callable[["OperationSignature"], "bool | tuple[bool, str]"]
ImplementationFunction = Callable[..., Any]

_CAPABILITY = _lib.CAPABILITY_FN


@dataclasses.dataclass(frozen=True, slots=True)
class OperationSignature:
    operation: str
    device_type: str
    architecture: str
    dtype: str
    shape: tuple[int, ...]
    layout: str
    mode: str
    mask: str
    inplace: bool
    attributes: tuple[tuple[str, str], ...] = ()
    strides: tuple[int, ...] = ()

    @classmethod
    def create(cls, *, operation: str, device_type: str, architecture: str, dtype: str,
               shape, layout: str = "contiguous", mode: str = "inference", mask: str = "none",
               inplace: bool = False, attributes: Mapping[str, Any] | None = None,
               strides=()) -> "OperationSignature":
        normalized = tuple(sorted((str(k), str(v)) for k, v in (attributes or {}).items()))
        return cls(operation=operation, device_type=device_type, architecture=architecture,
                   dtype=dtype, shape=tuple(int(v) for v in shape), layout=layout, mode=mode,
                   mask=mask, inplace=bool(inplace), attributes=normalized,
                   strides=tuple(int(v) for v in strides))

    def as_dict(self) -> dict[str, Any]:
        result = dataclasses.asdict(self)
        result["shape"] = list(self.shape)
        result["strides"] = list(self.strides)
        result["attributes"] = dict(self.attributes)
        return result

    def canonical_json(self) -> str:
        return json.dumps(self.as_dict(), sort_keys=True)


@dataclasses.dataclass(frozen=True, slots=True)
class OperationImplementation:
    operation: str
    name: str
    function: ImplementationFunction
    supports: Capability
    priority: int
    version: str


@dataclasses.dataclass(frozen=True, slots=True)
class Selection:
    implementation: OperationImplementation | None
    rejected: tuple[tuple[str, str], ...]
    cache_hit: bool


class _Interrupted(Exception):
    pass


class PolicyCore:
    """The C++ policy core with the method surface of the reference's PyO3
    bridge class ``OperatorRegistry`` (``crates/fireprot-bridge/src/lib.rs:
    86-125``): JSON metadata / signatures in, JSON selections / manifests out;
    capability callbacks take the signature JSON and return ``bool`` or
    ``(bool, reason)``. An ``Exception`` inside a callback rejects that
    candidate; ``KeyboardInterrupt`` / ``SystemExit`` escape the resolution,
    which is then neither cached nor counted (``lib.rs:42-58``)."""

    ABI_VERSION = 1

    def __init__(self) -> None:
        self._lib = _lib.load()
        self._core = self._lib.fpb_registry_new()
        if not self._core:
            raise MemoryError("fpb_registry_new failed")
        self._callbacks: dict[tuple[str, str], Any] = {}
        self._pending: BaseException | None = None

    def __del__(self):
        core = getattr(self, "_core", None)
        if core:
            self._lib.fpb_registry_free(core)
            self._core = None

    def _wrap(self, capability):
        def call(signature_json, _user, reason_buf, cap):
            try:
                value = capability(signature_json.decode())
                if isinstance(value, tuple):
                    if len(value) != 2:
                        raise ValueError("capability tuple must have two items")
                    ok, reason = bool(value[0]), str(value[1])
                else:
                    ok, reason = bool(value), "capability returned false"
            except Exception as error:  # rejects only this candidate
                ok, reason = False, f"capability error: {error}"
            except BaseException as error:  # KeyboardInterrupt / SystemExit escape
                self._pending = error
                return -1
            if not ok:
                data = reason.encode()[: max(0, cap - 1)]
                ctypes.memmove(reason_buf, data + b"\0", len(data) + 1)
            return 1 if ok else 0
        return _CAPABILITY(call)

    def register(self, metadata: str, supports) -> None:
        if not callable(supports):
            raise TypeError("supports must be callable")
        meta = json.loads(metadata)
        cb = self._wrap(supports)
        rc = self._lib.fpb_registry_register(self._core, metadata.encode(), cb, None)
        if rc == 2:
            raise ValueError("operation, implementation name and version must not be empty")
        if rc == 3:
            raise ValueError("implementation name is already registered for this operation")
        if rc != 0:
            raise ValueError(f"invalid implementation metadata ({rc})")
        self._callbacks[(meta["operation"], meta["name"])] = cb

    def unregister(self, operation: str, name: str) -> None:
        rc = self._lib.fpb_registry_unregister(self._core, operation.encode(), name.encode())
        if rc == 5:
            raise KeyError("implementation is not registered for this operation")
        if rc != 0:
            raise ValueError(f"unregister failed ({rc})")
        self._callbacks.pop((operation, name), None)

    def resolve(self, signature: str) -> str:
        buf = ctypes.create_string_buffer(1 << 16)
        self._pending = None
        rc = self._lib.fpb_registry_resolve(self._core, signature.encode(), buf, len(buf))
        if rc == 6:
            pending, self._pending = self._pending, None
            raise pending if pending is not None else _Interrupted("capability interrupted")
        if rc != 0:
            raise ValueError(f"registry resolution failed ({rc})")
        return buf.value.decode()

    def manifest(self) -> str:
        size = 1 << 16
        while True:
            buf = ctypes.create_string_buffer(size)
            rc = self._lib.fpb_registry_manifest(self._core, buf, size)
            if rc == 0:
                return buf.value.decode()
            if rc > 0:
                raise ValueError(f"manifest failed ({rc})")
            size = -rc + 1024

    def clear_runtime_state(self) -> None:
        self._lib.fpb_registry_clear_runtime_state(self._core)


class OperationRegistry:
    """Thread-safe registry whose missing match always means native fallback
    (``python/fireprot/ops/registry.py:90-175``)."""

    def __init__(self) -> None:
        self._functions: dict[tuple[str, str], OperationImplementation] = {}
        self._policy = PolicyCore()
        self._lock = threading.RLock()

    def register(self, *, operation: str, name: str, function: ImplementationFunction,
                 supports: Capability, priority: int = 0,
                 version: str = "1") -> OperationImplementation:
        implementation = OperationImplementation(operation=operation, name=name,
                                                 function=function, supports=supports,
                                                 priority=int(priority), version=str(version))
        if not callable(function) or not callable(supports):
            raise TypeError("function and supports must be callable")

        def capability(signature_json: str):
            return supports(OperationSignature.create(**json.loads(signature_json)))

        with self._lock:
            self._policy.register(json.dumps({"operation": operation, "name": name,
                                              "priority": implementation.priority,
                                              "version": implementation.version}), capability)
            self._functions[(operation, name)] = implementation
        return implementation

    def unregister(self, operation: str, name: str) -> None:
        with self._lock:
            self._policy.unregister(operation, name)
            del self._functions[(operation, name)]

    def resolve(self, signature: OperationSignature) -> Selection:
        with self._lock:
            selected = json.loads(self._policy.resolve(signature.canonical_json()))
            meta = selected["implementation"]
            impl = (self._functions[(meta["operation"], meta["name"])]
                    if meta is not None else None)
            return Selection(impl, tuple((r["implementation"], r["reason"])
                                         for r in selected["rejected"]), selected["cache_hit"])

    def dispatch(self, signature: OperationSignature, fallback: ImplementationFunction,
                 *args: Any, **kwargs: Any) -> Any:
        selection = self.resolve(signature)
        function = (selection.implementation.function
                    if selection.implementation is not None else fallback)
        return function(*args, **kwargs)

    def manifest(self) -> dict[str, Any]:
        with self._lock:
            result = json.loads(self._policy.manifest())
        result["policy_engine"] = {"name": "fireprot-b200-core", "library": str(_lib.LIB_PATH),
                                   "bridge_abi": PolicyCore.ABI_VERSION}
        return result

    def clear_runtime_state(self) -> None:
        with self._lock:
            self._policy.clear_runtime_state()


_registry = None
_registry_lock = threading.Lock()


def get_registry() -> OperationRegistry:
    """The process-wide registry (created on first use)."""
    global _registry
    with _registry_lock:
        if _registry is None:
            _registry = OperationRegistry()
        return _registry


def signature_from_tensor(operation: str, tensor: Any, *, architecture: str, mode: str, mask: str,
                          inplace: bool, attributes: Mapping[str, Any] | None = None
                          ) -> OperationSignature:
    layout = "contiguous" if tensor.is_contiguous() else "strided"
    return OperationSignature.create(
        operation=operation, device_type=tensor.device.type, architecture=architecture,
        dtype=str(tensor.dtype).removeprefix("torch."), shape=tuple(tensor.shape),
        strides=tuple(tensor.stride()), layout=layout, mode=mode, mask=mask, inplace=inplace,
        attributes=attributes)


def __getattr__(name: str):
    # ``registry`` is created on first access (it needs the C++ core)
    if name == "registry":
        return get_registry()
    raise AttributeError(name)
