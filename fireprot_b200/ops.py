"""Torch-facing wrappers of the C-ABI entry points.

Each wrapper validates its tensors, allocates outputs and the workspace with
torch on the current stream (as the reference's ``lt_bmm.py:70-74`` does) and
raises on any non-zero status. CPU tensors are rejected: there is no CPU
fallback in this package.
"""
from __future__ import annotations

import torch

from . import _lib

STRICT, FAST = 0, 1
_PRECISIONS = {"strict": STRICT, "fast": FAST, STRICT: STRICT, FAST: FAST}


def precision_code(precision) -> int:
    try:
        return _PRECISIONS[precision]
    except KeyError:
        raise ValueError(f"precision must be 'strict' or 'fast', got {precision!r}") from None


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors):
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("fireprot_b200 ops take CUDA tensors only (no CPU fallback)")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def workspace_status(ws: torch.Tensor) -> int:
    """Synchronise and read the device status word (0 = every wait completed)."""
    lib = _lib.load()
    out = _lib.c_int(0)
    _lib.check(lib.fpb_workspace_status(ws.data_ptr(), _stream_ptr(ws.device), out),
               "fpb_workspace_status")
    return out.value


def packed_bmm(a: torch.Tensor, b: torch.Tensor, outgoing: bool, precision="strict",
               return_workspace: bool = False):
    """``bmm(a, b^T)`` (outgoing) or ``bmm(a^T, b)`` (incoming) over
    ``[batch, n, n]`` FP32 planes, on tcgen05 tensor cores."""
    _require_cuda(a, b)
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise RuntimeError("packed_bmm takes float32 planes")
    if a.shape != b.shape or a.ndim != 3 or a.shape[1] != a.shape[2]:
        raise RuntimeError("packed_bmm takes two [batch, n, n] planes")
    a, b = a.contiguous(), b.contiguous()
    lib = _lib.load()
    p = precision_code(precision)
    batch, n = a.shape[0], a.shape[1]
    out = torch.empty_like(a)
    ws = workspace(lib.fpb_packed_bmm_workspace_size(batch, n, p), a.device)
    _lib.check(lib.fpb_packed_bmm(a.data_ptr(), b.data_ptr(), out.data_ptr(), batch, n,
                                  int(bool(outgoing)), p, ws.data_ptr(), ws.numel(),
                                  _stream_ptr(a.device)), "fpb_packed_bmm")
    return (out, ws) if return_workspace else out
