# Portions of this file (the source-pinned scope `attention_scope`, the
# dispatcher call contract in `contract_ok` and `AttentionDispatcher.__call__`)
# follow FireProt's OpenFold3 adapter, python/fireprot/adapters/openfold3/
# attention.py, which carries this notice:
#
#   Copyright 2026 AlQuraishi Laboratory
#   Copyright 2026 Outpace Bio, Inc.
#   Copyright 2026 Advanced Micro Devices, Inc.
#   Copyright 2025 NVIDIA Corporation
#   Copyright 2021 DeepMind Technologies Limited
#
#   Licensed under the Apache License, Version 2.0 (the "License");
#   you may not use this file except in compliance with the License.
#   You may obtain a copy of the License at
#
#       http://www.apache.org/licenses/LICENSE-2.0
#
#   Unless required by applicable law or agreed to in writing, software
#   distributed under the License is distributed on an "AS IS" BASIS,
#   WITHOUT WARRANTIES OR CONDITIONS OF ANY KIND, either express or implied.
#   See the License for the specific language governing permissions and
#   limitations under the License.
#
# Modified here: the scope dispatches to the B200 attention core
# (fpb_attention_core) instead of a HIP softmax, the installation is an
# object with explicit arm/disarm, and the device contract accepts any N.
# This file, including these modifications, is Apache-2.0.

"""OpenFold3 ``_attention`` scope for the B200 backend.

The reference's OpenFold3 ``hip_fused`` worker replaces
``openfold3.core.model.primitives.attention._attention`` inside a scope
(``python/fireprot/adapters/openfold3/attention.py:43-148``): the upstream
function keeps running for every call the dispatcher does not accept, and
only the thread (context) that opened the scope sees the replacement. Its
accepted calls run QK on upstream einsum, mask + bias + softmax on a HIP
kernel (``backends/amd/softmax_fp32.py:19-84``), and PV on upstream einsum.

Here an accepted call runs the whole of it on the B200 attention core
(``fpb_attention_core``: ``softmax(q k^T + mask + bias) v`` in one kernel,
q pre-scaled by the caller as upstream does): q, k, v ``[B, 4, N, 32]``,
``biases = [mask [B|1, 1, 1, N], bias [1, 4, N, N]]``, FP32 on the GPU, any
non-negative strides, any N. The result is ``[B, 4, N, 32]`` (a transposed
view of the kernel's ``[B, N, 4, 32]`` output, which is the layout the
upstream caller transposes to next).

Same interface as the reference module: ``attention_scope(dispatcher)``,
``_scoped_hook(module, dispatcher)``, ``AttentionDispatcher(kernel)`` with
``kernel=None`` meaning native-only dispatch, and ``manifest()``.
"""
from __future__ import annotations

import hashlib
import threading
from contextlib import contextmanager
from contextvars import ContextVar
from pathlib import Path

import torch

from . import _lib, backend, ops
from .registry import OperationRegistry, signature_from_tensor

# The upstream file the scope was validated against (the reference pins the
# same OpenFold3 source, adapters/openfold3/attention.py:37).
SOURCE_SHA256 = "30fe5433982ee73e3d7ce5341fa6b510b1ea332dbde072d56129632cc53f0746"
IMPL = "b200_attention_core"

_active_dispatcher: ContextVar = ContextVar("fireprot_b200_openfold3_attention", default=None)
_guard = threading.RLock()
_holder = [None]  # the one live installation, or None


class _Installation:
    """``module._attention`` replaced by a trampoline that asks the calling
    context for its dispatcher. The trampoline stays valid after the scope
    ends (a caller may have kept a reference to it): once disarmed it always
    calls the original."""

    def __init__(self, module, dispatcher):
        self.module = module
        self.original = module._attention
        self.armed = True
        self.token = None

        def trampoline(*args, **kwargs):
            dispatcher_here = _active_dispatcher.get()
            if self.armed and dispatcher_here is not None:
                return dispatcher_here(self.original, *args, **kwargs)
            return self.original(*args, **kwargs)

        self.trampoline = trampoline
        self.dispatcher = dispatcher

    def arm(self):
        self.module._attention = self.trampoline
        self.token = _active_dispatcher.set(self.dispatcher)

    def disarm(self):
        """Restore the original unless a third party replaced the hook, in
        which case its replacement stays and this raises."""
        self.armed = False
        _active_dispatcher.reset(self.token)
        if self.module._attention is not self.trampoline:
            raise RuntimeError("OpenFold3 attention hook changed during its scope")
        self.module._attention = self.original


@contextmanager
def _scoped_hook(module, dispatcher):
    """Install ``dispatcher`` as ``module._attention`` for the calling
    context only. Other threads and contexts, and calls made after the scope
    closed through a reference taken inside it, reach the original function.
    A second scope (nested or from another thread) is refused; the guard is
    released on every exit path, including a failed restore."""
    with _guard:
        if _holder[0] is not None:
            raise RuntimeError("An OpenFold3 attention scope is already installed")
        inst = _Installation(module, dispatcher)
        inst.arm()
        _holder[0] = inst
    try:
        yield
    finally:
        with _guard:
            _holder[0] = None
            inst.disarm()


@contextmanager
def attention_scope(dispatcher):
    """Scope over the pinned upstream OpenFold3 attention module."""
    import openfold3.core.model.primitives.attention as module  # upstream, when installed
    source = Path(module.__file__).resolve()
    if hashlib.sha256(source.read_bytes()).hexdigest() != SOURCE_SHA256:
        raise RuntimeError("Unsupported OpenFold3 attention source")
    function = module._attention
    code = getattr(function, "__code__", None)
    if (code is None or code.co_name != "_attention"
            or Path(code.co_filename).resolve() != source):
        raise RuntimeError("OpenFold3 attention was already replaced")
    with _scoped_hook(module, dispatcher):
        yield


class AttentionCoreKernel:
    """The B200 attention core bound to one device, with the kernel-object
    surface the dispatcher expects (``device``, ``supports``, ``receipt``,
    ``launches_submitted``)."""

    def __init__(self, device=None):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA GPU unavailable")
        self.device = torch.cuda.current_device() if device is None else int(device)
        lib = _lib.load()  # raises when the library is missing
        if lib.fpb_device_supported(self.device) != 0:
            raise RuntimeError("the B200 attention core needs an sm_100 device")
        self.receipt = {"library": str(_lib.LIB_PATH), "abi": lib.fpb_abi_version(),
                        "entry": "fpb_attention_core"}
        self.launches_submitted = 0

    def supports(self, query, key, value, biases) -> bool:
        return compatible_tensors(query, key, value, biases) and query.device.index == self.device

    def __call__(self, query, key, value, biases, precision="strict"):
        if not self.supports(query, key, value, biases):
            raise ValueError("Unsupported attention tensors or device")
        with torch.cuda.device(self.device):
            # a row with no finite logit is NaN, as upstream's softmax and the
            # reference's kernel give it (fireprot_softmax_fp32.cpp:61-62)
            out = ops.attention_core(query, key, value, list(biases), precision=precision,
                                     empty_rows="nan")
        self.launches_submitted += 1
        return out.transpose(1, 2)  # [B, N, 4, 32] storage, [B, 4, N, 32] view


def contract_ok(query, key, value, biases) -> bool:
    """Shapes, dtype and strides of an accepted call (device not checked)."""
    if not isinstance(biases, (tuple, list)) or len(biases) != 2:
        return False
    tensors = (query, key, value, *biases)
    if any(type(t) is not torch.Tensor for t in tensors):
        return False
    if any(t.dtype != torch.float32 or t.requires_grad or t.is_neg() or t.is_conj()
           for t in tensors):
        return False
    if (query.ndim != 4 or query.shape != key.shape or query.shape != value.shape
            or query.shape[0] < 1 or query.shape[1] != 4 or query.shape[2] < 1
            or query.shape[3] != 32):
        return False
    mask, bias = biases
    n = query.shape[2]
    return (mask.ndim == bias.ndim == 4
            and mask.shape[0] in (1, query.shape[0])
            and tuple(mask.shape[1:]) == (1, 1, n)
            and tuple(bias.shape) == (1, 4, n, n)
            and all(st >= 0 for t in tensors for st in t.stride()))


def compatible_tensors(query, key, value, biases) -> bool:
    """The contract plus: every tensor on the query's CUDA device."""
    return (contract_ok(query, key, value, biases)
            and all(t.is_cuda and t.device == query.device
                    for t in (query, key, value, *biases)))


class AttentionDispatcher:
    """Dispatcher for ``attention_scope``. ``kernel``: an
    :class:`AttentionCoreKernel`, or None for native-only dispatch."""

    def __init__(self, kernel):
        self.kernel = kernel
        self.registry = OperationRegistry()
        self.registry.register(
            operation="attention", name=IMPL, function=self._fused,
            priority=backend.PRIORITY, version="attention-core-v1",
            supports=lambda signature: (
                dict(signature.attributes).get("eligible") == "True",
                "FP32 GPU tensor, mask, bias or layout outside the attention-core contract"))

    def _eligible(self, query, key, value, biases) -> bool:
        if self.kernel is None or torch.is_grad_enabled():
            return False
        return bool(self.kernel.supports(query, key, value, biases))

    def __call__(self, native, query, key, value, biases, use_high_precision=False):
        if type(query) is not torch.Tensor:
            return native(query, key, value, biases, use_high_precision=use_high_precision)
        eligible = self._eligible(query, key, value, biases)
        signature = signature_from_tensor(
            "attention", query,
            architecture=(backend.device_architecture(query) if self.kernel is not None
                          else "unknown"),
            mode="training" if torch.is_grad_enabled() else "inference",
            mask="pair_and_token", inplace=False,
            attributes={"eligible": eligible, "high_precision": use_high_precision})
        return self.registry.dispatch(signature, native, query, key, value, biases,
                                      use_high_precision=use_high_precision)

    def _fused(self, query, key, value, biases, use_high_precision=False):
        # high precision always runs strict (3xTF32); otherwise the backend's mode
        precision = "strict" if use_high_precision else backend.get_precision()
        return self.kernel(query, key, value, biases, precision=precision).to(query.dtype)

    def manifest(self):
        return dict(registry=self.registry.manifest(),
                    kernel=None if self.kernel is None else self.kernel.receipt,
                    launches_submitted=(0 if self.kernel is None
                                        else self.kernel.launches_submitted),
                    limits=["Registry selection counts precede the launch and do not prove "
                            "that the kernel completed; a non-zero C-ABI status raises."])
