"""ESMFold2 triangle contraction on the B200 backend.

The reference's ESMFold2 candidate replaces the bound method
``TriangleMultiplicativeBlock._triangular_contract_chunked(left, right,
chunk_size)`` of selected blocks of a loaded model inside a scope
(``python/fireprot/adapters/esmfold2/triangle.py:36-106``): outgoing
``x_ijc = sum_k l_ikc r_jkc``, incoming ``x_ijc = sum_k l_kic r_kjc`` on
``[1, n, n, C]`` channels-last FP32 tensors (C = 256 in ESMFold2). Here an
accepted call is one ``fpb_triangle_contract`` (3xTF32 tensor cores in the
strict mode, BF16 operands in the fast mode); everything else, including any
call under autocast or with autograd, runs the model's own method.

Same interface as the reference module: ``triangle_scope(model)`` yields a
``TriangleDispatcher`` whose ``manifest()`` reports the dispatch decisions.
"""
from __future__ import annotations

import hashlib
import types
from contextlib import contextmanager
from pathlib import Path

import torch

from . import backend, ops
from .registry import OperationRegistry, signature_from_tensor

# The upstream ESMFold2 layers file the scope was validated against (the
# reference pins the same source, adapters/esmfold2/triangle.py:16).
LAYERS_SHA256 = "35f25607bd789d36fb4f46e184c3ac09f3c435538806d3531f42525bbdc372f2"
OPERATION = "esmfold2_triangle_contract"
IMPL = "b200_triangle_contract"
METHOD = "_triangular_contract_chunked"
# model sub-trees whose triangle blocks are replaced (the reference's scope)
PREFIXES = ("folding_trunk.", "lm_encoder.", "parcae_coda.", "confidence_head.folding_trunk.",
            "msa_encoder.")


def eligible(left, right, flow) -> bool:
    """Calls the B200 contraction accepts."""
    if type(left) is not torch.Tensor or type(right) is not torch.Tensor:
        return False
    if torch.is_grad_enabled() or torch.is_autocast_enabled("cuda"):
        return False
    if flow not in ("outgoing", "incoming"):
        return False
    if not (left.is_cuda and right.device == left.device):
        return False
    if backend.device_architecture(left) != backend.ARCHITECTURE:
        return False
    if left.dtype != torch.float32 or right.dtype != torch.float32:
        return False
    if any(t.requires_grad or t.is_conj() or t.is_neg() for t in (left, right)):
        return False
    return (left.ndim == 4 and left.shape == right.shape and left.shape[0] == 1
            and left.shape[1] == left.shape[2] and left.shape[3] % 32 == 0)


class TriangleDispatcher:
    """Registry-gated replacement of the chunked contraction."""

    def __init__(self):
        self.registry = OperationRegistry()
        self.calls = 0
        self.registry.register(
            operation=OPERATION, name=IMPL, function=self._run, priority=backend.PRIORITY,
            version="tricontract-v1",
            supports=lambda s: (dict(s.attributes).get("eligible") == "True",
                                "tensor, dtype, layout, autocast, autograd or device outside "
                                "the B200 contraction"))

    def _run(self, left, right, chunk_size, flow):
        del chunk_size  # the chunking of the native loop only bounds its memory
        self.calls += 1
        return ops.triangle_contract(left, right, outgoing=flow == "outgoing",
                                     precision=backend.get_precision())

    def __call__(self, native, left, right, chunk_size, flow):
        if type(left) is not torch.Tensor or type(right) is not torch.Tensor:
            return native(left, right, chunk_size)
        ok = eligible(left, right, flow)
        sig = signature_from_tensor(
            OPERATION, left,
            architecture=backend.device_architecture(left) if left.is_cuda else "cpu",
            mode="training" if torch.is_grad_enabled() else "inference",
            mask="already_applied", inplace=False,
            attributes=dict(eligible=ok, flow=flow, chunk_size=chunk_size,
                            right_strides=tuple(right.stride()),
                            autocast=(str(torch.get_autocast_dtype("cuda"))
                                      if torch.is_autocast_enabled("cuda") else "off")))
        return self.registry.dispatch(sig, lambda a, b, c, _flow: native(a, b, c),
                                      left, right, chunk_size, flow)

    def manifest(self):
        return dict(implementation=IMPL, completed_dispatches=self.calls,
                    registry=self.registry.manifest(),
                    scope="triangle contractions of the trunk, LM encoder, coda, confidence "
                          "and MSA blocks; the diffusion module is unchanged")


def _install(model, block_type, dispatcher):
    """Bind a dispatching method on every matching block; returns the list
    of (block, replacement) installed."""
    installed = []
    for name, block in model.named_modules():
        if type(block) is not block_type or not name.startswith(PREFIXES):
            continue
        if METHOD in block.__dict__:
            raise RuntimeError("ESMFold2 contraction already replaced")
        original = getattr(block, METHOD)

        def contract(self, left, right, chunk_size, _original=original):
            return dispatcher(_original, left, right, chunk_size, self.flow)

        bound = types.MethodType(contract, block)
        setattr(block, METHOD, bound)
        installed.append((block, bound))
    return installed


def _uninstall(installed):
    for block, bound in reversed(installed):
        if getattr(block, METHOD) is not bound:
            raise RuntimeError("ESMFold2 triangle hook changed during scope")
        delattr(block, METHOD)


@contextmanager
def patched_blocks(model, block_type):
    """The scope over an explicit block class (used by ``triangle_scope``)."""
    dispatcher = TriangleDispatcher()
    installed = []
    try:
        installed = _install(model, block_type, dispatcher)
        if not installed:
            raise RuntimeError("No compatible ESMFold2 triangle modules")
        yield dispatcher
    finally:
        _uninstall(installed)


@contextmanager
def triangle_scope(model):
    """Scope over the pinned upstream ESMFold2 layers module."""
    import esm.models.esmfold2.layers as layers  # upstream, when installed
    source = Path(layers.__file__).resolve()
    if hashlib.sha256(source.read_bytes()).hexdigest() != LAYERS_SHA256:
        raise RuntimeError("Unsupported ESMFold2 triangle source")
    with patched_blocks(model, layers.TriangleMultiplicativeBlock) as dispatcher:
        yield dispatcher
