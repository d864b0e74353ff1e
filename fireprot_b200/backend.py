"""The ``b200`` backend: capability-gated dispatch entry points with the
reference's signatures, registered beside its ``native`` / ``hip_fused``
choices.

Entry points (same keyword signatures as the reference's AMD backend):

- ``dispatch_triangle_multiplication(*, module, z, mask, inplace_safe,
  add_with_inplace, inplace_chunk_size, native)``
  (``python/fireprot/backends/amd/triangle_multiplication.py:389-430``);
- ``dispatch_triangle_attention(*, module, q, k, v, biases, native)``
  (``python/fireprot/backends/amd/triangle_attention.py:199-256``);
- ``dispatch_transition(*, module, x, native)``
  (``python/fireprot/backends/amd/recycle.py:360``);
- ``transpose_pair(x, *, training)`` (``pair_layout.py:8-26``);
- ``triangle_attention_module(*, module, z, mask, starting, native)``: the
  module-level fused triangle attention (LN + projections + attention + gate
  + output), the boundary AtlasFold's runtime hooks use
  (``adapters/atlasfold/runtime.py:145-157``).

Each builds an ``OperationSignature`` and dispatches through the registry;
a rejected signature runs the caller's ``native``. After a launch there is no
fallback: a non-zero C-ABI status raises (``lt_bmm.py:76-82``).

Precision: ``FIREPROT_B200_PRECISION`` (``strict`` default, or ``fast``) at
import, or :func:`set_precision`.
"""
from __future__ import annotations

import os
import threading
from collections.abc import Callable, Sequence
from typing import Any

import torch

from . import _lib, ops
from .registry import OperationSignature, get_registry, signature_from_tensor

BACKEND = "b200"
ARCHITECTURE = "sm_100"
TRIMUL = "triangle_multiplication"
TRIATT = "triangle_attention"
TRIATT_MODULE = "triangle_attention_module"
TRANSITION = "gated_transition"

TRIMUL_IMPL = "b200-sm100-fused-triangle-multiplication"
TRIATT_IMPL = "b200-sm100-attention-core"
TRIATT_MODULE_IMPL = "b200-sm100-fused-triangle-attention"
TRANSITION_IMPL = "b200-sm100-fused-transition"
PRIORITY = 50  # above every reference AMD candidate (<= 40)

_registered = False
_precision = os.environ.get("FIREPROT_B200_PRECISION", "strict")
_counts_lock = threading.Lock()
_counts: dict[str, int] = {}


def set_precision(precision: str) -> None:
    """Select ``strict`` (3xTF32) or ``fast`` (BF16 operands) for new calls."""
    global _precision
    ops.precision_code(precision)
    _precision = precision


def get_precision() -> str:
    return _precision


def _count(name: str) -> None:
    with _counts_lock:
        _counts[name] = _counts.get(name, 0) + 1


def manifest() -> dict[str, Any]:
    """Backend counters plus the registry's policy manifest."""
    with _counts_lock:
        counts = dict(_counts)
    return {"backend": BACKEND, "precision": _precision, "counts": counts,
            "operations": get_registry().manifest()}


def device_architecture(tensor: Any) -> str:
    try:
        major, minor = torch.cuda.get_device_capability(tensor.device)
        return f"sm_{major}{minor}"
    except Exception:
        return "unknown"


def _mode(module: Any, *tensors: Any) -> str:
    """``inference`` only without training mode, autograd or grad-requiring
    inputs (``triangle_multiplication.py:399-404``)."""
    if (getattr(module, "training", False) or torch.is_grad_enabled()
            or any(getattr(t, "requires_grad", False) for t in tensors)):
        return "training"
    return "inference"


def _library_available() -> bool:
    try:
        _lib.load()
        return True
    except Exception:
        return False


def _common(sig: OperationSignature):
    if sig.device_type != "cuda":
        return False, "device is not CUDA"
    if sig.architecture != ARCHITECTURE:
        return False, f"architecture is not {ARCHITECTURE}"
    if sig.dtype != "float32":
        return False, "dtype is not float32"
    if sig.mode != "inference":
        return False, "training or autograd is enabled"
    if not _library_available():
        return False, "fireprot_b200 CUDA library is unavailable"
    return True


def _cuda_f32(t) -> bool:
    return t is not None and t.is_cuda and t.dtype == torch.float32


# ---------------------------------------------------------------- TriMul
def _trimul_weights(module) -> dict | None:
    try:
        linears = {k: getattr(module, name) for k, name in (
            ("w_a_p", "linear_a_p"), ("w_a_g", "linear_a_g"), ("w_b_p", "linear_b_p"),
            ("w_b_g", "linear_b_g"), ("w_g", "linear_g"), ("w_z", "linear_z"))}
        if any(getattr(lin, "bias", None) is not None for lin in linears.values()):
            return None
        w = {k: lin.weight for k, lin in linears.items()}
        w.update(ln_in_w=module.layer_norm_in.weight, ln_in_b=module.layer_norm_in.bias,
                 ln_out_w=module.layer_norm_out.weight, ln_out_b=module.layer_norm_out.bias)
    except AttributeError:
        return None
    if not all(_cuda_f32(t) for t in w.values()):
        return None
    if any(tuple(w[k].shape) != (128, 128) for k in ("w_a_p", "w_a_g", "w_b_p", "w_b_g", "w_g",
                                                       "w_z")):
        return None
    return w


def _supports_trimul(sig: OperationSignature):
    ok = _common(sig)
    if ok is not True:
        return ok
    a = dict(sig.attributes)
    if sig.layout != "contiguous":
        return False, "input is not contiguous"
    if not sig.inplace:
        return False, "the fused path updates z in place (inplace_safe required)"
    if len(sig.shape) != 3 or sig.shape[0] != sig.shape[1] or sig.shape[2] != 128:
        return False, "only unbatched [N, N, 128] pair tensors are supported"
    if a.get("c_z") != "128" or a.get("c_hidden") != "128":
        return False, "c_z and c_hidden must both be 128"
    if sig.mask not in ("none", "dense"):
        return False, "only absent or dense pair masks are supported"
    if a.get("weights") != "ok":
        return False, "weights are not bias-free CUDA float32 [128, 128] linears"
    return True


def _b200_trimul(*, module, z, mask, inplace_safe, add_with_inplace, inplace_chunk_size,
                 native):
    del inplace_safe, inplace_chunk_size, native
    w = _trimul_weights(module)
    m = None if mask is None else mask.to(torch.float32).contiguous()
    eps = float(getattr(module.layer_norm_in, "eps", 1e-5))
    ops.trimul(z, m, w, outgoing=bool(module._outgoing), add=bool(add_with_inplace),
               precision=_precision, eps=eps)
    _count(TRIMUL_IMPL)
    return z


def dispatch_triangle_multiplication(*, module: Any, z: Any, mask: Any, inplace_safe: bool,
                                     add_with_inplace: bool, inplace_chunk_size: int | None,
                                     native: Callable[..., Any]) -> Any:
    """Protenix ``TriangleMultiplicativeUpdate`` boundary: returns ``z``
    updated in place (``z + delta`` or ``delta``)."""
    weights_ok = _trimul_weights(module) is not None and (
        mask is None or (mask.is_cuda and tuple(mask.shape) == tuple(z.shape[:2])))
    sig = signature_from_tensor(
        TRIMUL, z, architecture=device_architecture(z), mode=_mode(module, z),
        mask="none" if mask is None else "dense", inplace=inplace_safe,
        attributes={"direction": "outgoing" if getattr(module, "_outgoing", True) else "incoming",
                    "add_with_inplace": add_with_inplace,
                    "c_z": getattr(module, "c_z", -1), "c_hidden": getattr(module, "c_hidden", -1),
                    "weights": "ok" if weights_ok else "unsupported", "backend": BACKEND})
    return get_registry().dispatch(sig, native, module=module, z=z, mask=mask,
                                   inplace_safe=inplace_safe, add_with_inplace=add_with_inplace,
                                   inplace_chunk_size=inplace_chunk_size, native=native)


# ---------------------------------------------------------------- TriAttn core
def _supports_attention_core(sig: OperationSignature):
    ok = _common(sig)
    if ok is not True:
        return ok
    a = dict(sig.attributes)
    if len(sig.shape) != 4:
        return False, "q must be [B, H, N, D]"
    b, h, n, d = sig.shape
    if h != 4 or d != 32:
        return False, "heads must be 4 and head_dim 32"
    shapes = a.get("bias_shapes")
    if shapes not in (repr(((b, 1, 1, n), (1, 4, n, n))), repr(((1, 4, n, n),))):
        return False, "biases must be [mask [B,1,1,N],] triangle [1,4,N,N]"
    if a.get("qkv_shapes_match") != "True":
        return False, "q, k and v shapes or devices differ"
    return True


def _b200_attention_core(*, module, q, k, v, biases, native):
    del module, native
    out = ops.attention_core(q, k, v, list(biases), precision=_precision)
    _count(TRIATT_IMPL)
    return out


def dispatch_triangle_attention(*, module: Any, q: Any, k: Any, v: Any, biases: Sequence[Any],
                                native: Callable[..., Any]) -> Any:
    """Protenix ``Attention`` boundary: returns ``[*, Q, H, D]``."""
    bias_shapes = tuple(tuple(int(x) for x in bb.shape) for bb in biases)
    match = all(t.shape == q.shape and t.device == q.device and t.dtype == q.dtype
                for t in (k, v)) and all(bb.device == q.device and bb.dtype == q.dtype
                                          for bb in biases)
    sig = signature_from_tensor(
        TRIATT, q, architecture=device_architecture(q), mode=_mode(module, q, k, v),
        mask=("triangle-bias" if len(biases) == 1 else "additive-mask-and-triangle-bias"
              if len(biases) == 2 else "unsupported"),
        inplace=False,
        attributes={"bias_count": len(biases), "bias_shapes": repr(bias_shapes),
                    "qkv_shapes_match": match, "backend": BACKEND,
                    "heads": q.shape[-3] if q.ndim >= 3 else -1,
                    "head_dim": q.shape[-1] if q.ndim else -1})
    return get_registry().dispatch(sig, native, module=module, q=q, k=k, v=v, biases=biases,
                                   native=native)


# ---------------------------------------------------------------- TriAttn module
def _triattn_weights(module) -> dict | None:
    try:
        mha = module.mha
        w = dict(ln_w=module.layer_norm.weight, ln_b=module.layer_norm.bias,
                 w_q=mha.linear_q.weight, w_k=mha.linear_k.weight, w_v=mha.linear_v.weight,
                 w_bias=module.linear.weight, w_g=mha.linear_g.weight,
                 b_g=getattr(mha.linear_g, "bias", None), w_o=mha.linear_o.weight,
                 b_o=getattr(mha.linear_o, "bias", None))
        if any(getattr(getattr(mha, n), "bias", None) is not None
               for n in ("linear_q", "linear_k", "linear_v")):
            return None
        if getattr(module.linear, "bias", None) is not None:
            return None
        if int(mha.no_heads) != 4 or int(mha.c_hidden) != 32 or float(module.inf) != 1e9:
            return None
    except AttributeError:
        return None
    if not all(t is None or _cuda_f32(t) for t in w.values()):
        return None
    return w


def _supports_triattn_module(sig: OperationSignature):
    ok = _common(sig)
    if ok is not True:
        return ok
    a = dict(sig.attributes)
    if sig.layout != "contiguous":
        return False, "input is not contiguous"
    if len(sig.shape) != 3 or sig.shape[0] != sig.shape[1] or sig.shape[2] != 128:
        return False, "only unbatched [N, N, 128] pair tensors are supported"
    if sig.mask not in ("none", "dense"):
        return False, "only absent or dense pair masks are supported"
    if a.get("weights") != "ok":
        return False, "module is not H=4, d=32, inf=1e9 with CUDA float32 weights"
    return True


def _b200_triattn_module(*, module, z, mask, starting, native):
    del native
    w = _triattn_weights(module)
    m = None if mask is None else mask.to(torch.float32).contiguous()
    delta = torch.empty_like(z)
    ops.triattn(z, m, w, starting=bool(starting), precision=_precision,
                eps=float(getattr(module.layer_norm, "eps", 1e-5)), delta_out=delta)
    _count(TRIATT_MODULE_IMPL)
    return delta


def triangle_attention_module(*, module: Any, z: Any, mask: Any, starting: bool,
                              native: Callable[..., Any]) -> Any:
    """Module-level triangle attention: returns the update ``delta`` (the
    upstream ``TriangleAttention.forward`` value) without modifying ``z``."""
    weights_ok = _triattn_weights(module) is not None and (
        mask is None or (mask.is_cuda and tuple(mask.shape) == tuple(z.shape[:2])))
    sig = signature_from_tensor(
        TRIATT_MODULE, z, architecture=device_architecture(z), mode=_mode(module, z),
        mask="none" if mask is None else "dense", inplace=False,
        attributes={"starting": bool(starting), "weights": "ok" if weights_ok else "unsupported",
                    "backend": BACKEND})
    return get_registry().dispatch(sig, native, module=module, z=z, mask=mask,
                                   starting=starting, native=native)


# ---------------------------------------------------------------- transition
def _transition_weights(module) -> dict | None:
    try:
        w = dict(ln_w=module.layernorm1.weight, ln_b=module.layernorm1.bias,
                 w_a=module.linear_no_bias_a.weight, w_b=module.linear_no_bias_b.weight,
                 w_out=module.linear_no_bias.weight)
        if any(getattr(getattr(module, n), "bias", None) is not None
               for n in ("linear_no_bias_a", "linear_no_bias_b", "linear_no_bias")):
            return None
    except AttributeError:
        return None
    if not all(_cuda_f32(t) for t in w.values()):
        return None
    if tuple(w["w_a"].shape) != (512, 128) or tuple(w["w_out"].shape) != (128, 512):
        return None
    return w


def _supports_transition(sig: OperationSignature):
    ok = _common(sig)
    if ok is not True:
        return ok
    if sig.layout != "contiguous":
        return False, "input is not contiguous"
    if not sig.shape or sig.shape[-1] != 128:
        return False, "last dimension is not 128"
    if dict(sig.attributes).get("weights") != "ok":
        return False, "transition is not 4x, bias-free, CUDA float32"
    return True


def _b200_transition(*, module, x, native):
    del native
    w = _transition_weights(module)
    delta = torch.empty_like(x)
    ops.transition(x, w, precision=_precision, eps=float(getattr(module.layernorm1, "eps", 1e-5)),
                   delta_out=delta)
    _count(TRANSITION_IMPL)
    return delta


def dispatch_transition(*, module: Any, x: Any, native: Callable[[], Any]) -> Any:
    """Protenix pair ``Transition`` boundary: returns the update (``x`` unchanged)."""
    sig = signature_from_tensor(
        TRANSITION, x, architecture=device_architecture(x), mode=_mode(module, x), mask="none",
        inplace=False,
        attributes={"expansion": getattr(module, "n", -1),
                    "weights": "ok" if _transition_weights(module) is not None else "unsupported",
                    "backend": BACKEND})
    # the reference's transition fallback takes no arguments (recycle.py:383-404)
    return get_registry().dispatch(sig, lambda **_: native(), module=module, x=x, native=native)


# ---------------------------------------------------------------- layout
def transpose_pair(x: Any, *, training: bool) -> Any:
    """Pair transpose for the ending-node passes. The fused B200 kernels read
    the transposed pair layout directly, so inference gets a view; training
    (and CPU tensors) keep the upstream contiguous copy."""
    view = x.transpose(-2, -3)
    if training or torch.is_grad_enabled() or not x.is_cuda:
        return view.contiguous()
    return view


def register_all() -> None:
    """Register the b200 candidates (idempotent)."""
    global _registered
    reg = get_registry()
    if _registered:
        return
    for op, name, fn, sup in ((TRIMUL, TRIMUL_IMPL, _b200_trimul, _supports_trimul),
                              (TRIATT, TRIATT_IMPL, _b200_attention_core,
                               _supports_attention_core),
                              (TRIATT_MODULE, TRIATT_MODULE_IMPL, _b200_triattn_module,
                               _supports_triattn_module),
                              (TRANSITION, TRANSITION_IMPL, _b200_transition,
                               _supports_transition)):
        try:
            reg.register(operation=op, name=name, function=fn, supports=sup, priority=PRIORITY,
                         version="1")
        except ValueError:
            pass  # already registered in this process
    _registered = True


register_all()
