"""Torch-facing wrappers of the C-ABI entry points.

Each wrapper validates its tensors, allocates outputs and the workspace with
torch on the current stream (as the reference's ``lt_bmm.py:70-74`` does) and
raises on any non-zero status. CPU tensors are rejected: there is no CPU
fallback in this package.
"""
from __future__ import annotations

import ctypes

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


def _f32(t, name, n=None):
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32")
    return t.contiguous()


def trimul(z: torch.Tensor, mask, w: dict, *, outgoing: bool, add: bool = True,
           precision="strict", eps: float = 1e-5, return_workspace: bool = False):
    """Triangle multiplicative update in place on ``z`` ``[n, n, 128]``.

    ``w`` holds ``ln_in_w, ln_in_b, w_a_p, w_a_g, w_b_p, w_b_g, w_g, ln_out_w,
    ln_out_b, w_z`` (torch Linear layouts). Returns ``z`` (same storage).
    """
    _require_cuda(z, mask)
    if z.dtype != torch.float32 or z.ndim != 3 or z.shape[0] != z.shape[1] or z.shape[2] != 128:
        raise RuntimeError("trimul takes a float32 [n, n, 128] pair tensor")
    if not z.is_contiguous() or z.data_ptr() % 16:
        raise RuntimeError("trimul needs a contiguous, 16-byte aligned z")
    n = z.shape[0]
    if mask is not None:
        if tuple(mask.shape) != (n, n):
            raise RuntimeError("mask must be [n, n]")
        mask = mask.to(torch.float32).contiguous()
    names = ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p", "w_b_g", "w_g", "ln_out_w",
             "ln_out_b", "w_z")
    ws_t = [_f32(w[k], k) for k in names]
    _require_cuda(*ws_t)
    lib = _lib.load()
    p = precision_code(precision)
    ws = workspace(lib.fpb_trimul_workspace_size(n, 128, p), z.device)
    _lib.check(lib.fpb_trimul(z.data_ptr(), 0 if mask is None else mask.data_ptr(), n, 128,
                              *[t.data_ptr() for t in ws_t], float(eps), int(bool(outgoing)),
                              int(bool(add)), p, ws.data_ptr(), ws.numel(),
                              _stream_ptr(z.device)), "fpb_trimul")
    return (z, ws) if return_workspace else z


TRIATTN_WEIGHTS = ("ln_w", "ln_b", "w_q", "w_k", "w_v", "w_bias", "w_g", "b_g", "w_o", "b_o")


def triattn(z: torch.Tensor, mask, w: dict, *, starting: bool = True, precision="strict",
            eps: float = 1e-5, return_workspace: bool = False, delta_out=None):
    """Triangle attention update added in place to ``z`` ``[n, n, 128]``
    (H=4, d=32). ``w`` holds ``ln_w, ln_b, w_q, w_k, w_v, w_bias, w_g, w_o``
    and optional ``b_g`` / ``b_o``. Returns ``z`` (same storage), or, when
    ``delta_out`` (a float32 tensor like ``z``) is given, writes the update
    there, leaves ``z`` unchanged and returns ``delta_out``."""
    _require_cuda(z, mask)
    if z.dtype != torch.float32 or z.ndim != 3 or z.shape[0] != z.shape[1] or z.shape[2] != 128:
        raise RuntimeError("triattn takes a float32 [n, n, 128] pair tensor")
    if not z.is_contiguous() or z.data_ptr() % 16:
        raise RuntimeError("triattn needs a contiguous, 16-byte aligned z")
    n = z.shape[0]
    if mask is not None:
        if tuple(mask.shape) != (n, n):
            raise RuntimeError("mask must be [n, n]")
        mask = mask.to(torch.float32).contiguous()
    ptrs = []
    keep = []
    for k in TRIATTN_WEIGHTS:
        t = w.get(k)
        if t is None:
            if k in ("b_g", "b_o"):
                ptrs.append(0)
                continue
            raise RuntimeError(f"missing weight {k}")
        t = _f32(t, k)
        _require_cuda(t)
        keep.append(t)
        ptrs.append(t.data_ptr())
    lib = _lib.load()
    p = precision_code(precision)
    ws = workspace(lib.fpb_triattn_workspace_size(n, 128, 4, 32, p, int(mask is not None)),
                   z.device)
    dptr = 0
    if delta_out is not None:
        if (delta_out.shape != z.shape or delta_out.dtype != torch.float32
                or not delta_out.is_contiguous() or delta_out.device != z.device):
            raise RuntimeError("delta_out must be a contiguous float32 tensor shaped like z")
        dptr = delta_out.data_ptr()
    _lib.check(lib.fpb_triattn(z.data_ptr(), dptr, 0 if mask is None else mask.data_ptr(), n,
                               128, 4, 32, *ptrs, float(eps), int(bool(starting)), p,
                               ws.data_ptr(), ws.numel(), _stream_ptr(z.device)), "fpb_triattn")
    res = z if delta_out is None else delta_out
    return (res, ws) if return_workspace else res


def transition(z: torch.Tensor, w: dict, *, precision="strict", eps: float = 1e-5,
               return_workspace: bool = False, delta_out=None):
    """Pair transition update added in place to ``z`` ``[..., 128]``; ``w``
    holds ``ln_w, ln_b, w_a, w_b, w_out`` (4x expansion). Returns ``z``, or
    writes the update alone to ``delta_out`` (``z`` unchanged) when given."""
    _require_cuda(z)
    if z.dtype != torch.float32 or z.shape[-1] != 128:
        raise RuntimeError("transition takes float32 [..., 128] rows")
    if not z.is_contiguous() or z.data_ptr() % 16:
        raise RuntimeError("transition needs a contiguous, 16-byte aligned z")
    ts = [_f32(w[k], k) for k in ("ln_w", "ln_b", "w_a", "w_b", "w_out")]
    _require_cuda(*ts)
    if tuple(ts[2].shape) != (512, 128) or tuple(ts[4].shape) != (128, 512):
        raise RuntimeError("transition supports c=128 with 4x expansion")
    lib = _lib.load()
    p = precision_code(precision)
    ws = workspace(lib.fpb_transition_workspace_size(128, 4, p), z.device)
    rows = z.numel() // 128
    dptr = 0
    if delta_out is not None:
        if (delta_out.shape != z.shape or delta_out.dtype != torch.float32
                or not delta_out.is_contiguous() or delta_out.device != z.device):
            raise RuntimeError("delta_out must be a contiguous float32 tensor shaped like z")
        dptr = delta_out.data_ptr()
    _lib.check(lib.fpb_transition(z.data_ptr(), dptr, rows, 128, 4, *[t.data_ptr() for t in ts],
                                  float(eps), p, ws.data_ptr(), ws.numel(),
                                  _stream_ptr(z.device)), "fpb_transition")
    res = z if delta_out is None else delta_out
    return (res, ws) if return_workspace else res


def attention_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, biases, *,
                   precision="strict", empty_rows: str = "zero",
                   return_workspace: bool = False):
    """``softmax(q k^T + sum(biases)) v`` at the reference's dispatch boundary.

    q (pre-scaled), k, v: ``[B, 4, N, 32]`` float32, any strides; ``biases``
    is ``[triangle_bias]`` or ``[mask_bias, triangle_bias]`` with
    ``mask_bias [B, 1, 1, N]`` (or ``[1, 1, 1, N]``, shared by every batch
    entry) and ``triangle_bias [1, 4, N, N]``, any non-negative strides. Returns
    ``[B, N, 4, 32]`` (``triangle_attention.py:129``).

    ``empty_rows``: the result of a query row whose every logit is -inf:
    ``"zero"`` as torch's scaled_dot_product_attention (the Protenix
    dispatch, ``triangle_attention.py:83-129``), ``"nan"`` as a softmax
    whose row sum is zero (the OpenFold3 contract,
    ``fireprot_softmax_fp32.cpp:61-62``).
    """
    if empty_rows not in ("zero", "nan"):
        raise ValueError(f"empty_rows must be 'zero' or 'nan', got {empty_rows!r}")
    _require_cuda(q, k, v, *biases)
    if q.ndim != 4 or q.shape[1] != 4 or q.shape[3] != 32 or q.shape != k.shape \
            or q.shape != v.shape:
        raise RuntimeError("attention_core takes q, k, v of shape [B, 4, N, 32]")
    batch, _, n, _ = q.shape
    if any(t.dtype != torch.float32 for t in (q, k, v, *biases)):
        raise RuntimeError("attention_core takes float32 tensors")
    if len(biases) == 1:
        mask_bias, tri = None, biases[0]
    elif len(biases) == 2:
        mask_bias, tri = biases
    else:
        raise RuntimeError("attention_core takes one or two biases")
    if tuple(tri.shape) != (1, 4, n, n):
        raise RuntimeError("triangle bias must be [1, 4, N, N]")
    if mask_bias is not None and (mask_bias.ndim != 4 or mask_bias.shape[0] not in (1, batch)
                                  or tuple(mask_bias.shape[1:]) != (1, 1, n)):
        raise RuntimeError("mask bias must be [B, 1, 1, N] or [1, 1, 1, N]")
    if any(st < 0 for t in (q, k, v, *biases) for st in t.stride()):
        raise RuntimeError("attention_core takes non-negative strides")
    lib = _lib.load()
    p = precision_code(precision)
    out = torch.empty(batch, n, 4, 32, dtype=torch.float32, device=q.device)
    ws = workspace(lib.fpb_attention_core_workspace_size(batch, n, 4, 32, p,
                                                         int(mask_bias is not None)), q.device)

    keep = []

    def strides(t, broadcast_batch=False):
        st = list(t.stride())
        if broadcast_batch:
            st[0] = 0  # one mask row for every batch entry
        arr = (ctypes.c_longlong * 4)(*st)
        keep.append(arr)
        return ctypes.cast(arr, ctypes.c_void_p)

    qs, ks, vs, ts = strides(q), strides(k), strides(v), strides(tri)
    ms = (strides(mask_bias, broadcast_batch=mask_bias.shape[0] == 1)
          if mask_bias is not None else None)
    _lib.check(lib.fpb_attention_core_ex(
        q.data_ptr(), qs, k.data_ptr(), ks, v.data_ptr(), vs, batch, n, 4, 32, tri.data_ptr(), ts,
        0 if mask_bias is None else mask_bias.data_ptr(), ms, out.data_ptr(), p,
        int(empty_rows == "nan"), ws.data_ptr(), ws.numel(), _stream_ptr(q.device)),
        "fpb_attention_core_ex")
    return (out, ws) if return_workspace else out


def pair_block_workspace(n: int, precision, with_mask: bool, device) -> torch.Tensor:
    lib = _lib.load()
    nbytes = lib.fpb_pair_block_workspace_size(n, precision_code(precision), int(with_mask))
    if nbytes == 0:
        raise RuntimeError(f"unsupported pair block size n={n}")
    return workspace(nbytes, device)


def pair_block(z: torch.Tensor, mask, c_weights, *, precision="strict", eps: float = 1e-5,
               workspace=None, return_workspace: bool = False):
    """Pair stack of one Pairformer block in place on ``z`` ``[n, n, 128]``.

    ``c_weights`` is a ``modules.PairBlockWeights`` ctypes struct (see
    ``PairformerPairBlock.c_weights``). ``workspace`` may be passed to reuse
    one allocation across blocks.
    """
    _require_cuda(z, mask)
    if z.dtype != torch.float32 or z.ndim != 3 or z.shape[0] != z.shape[1] or z.shape[2] != 128:
        raise RuntimeError("pair_block takes a float32 [n, n, 128] pair tensor")
    if not z.is_contiguous() or z.data_ptr() % 16:
        raise RuntimeError("pair_block needs a contiguous, 16-byte aligned z")
    n = z.shape[0]
    if mask is not None:
        if tuple(mask.shape) != (n, n) or mask.dtype != torch.float32 or not mask.is_contiguous():
            raise RuntimeError("mask must be a contiguous float32 [n, n] tensor")
    lib = _lib.load()
    p = precision_code(precision)
    ws = workspace if workspace is not None else pair_block_workspace(n, p, mask is not None,
                                                                      z.device)
    _lib.check(lib.fpb_pair_block(z.data_ptr(), 0 if mask is None else mask.data_ptr(), n,
                                  ctypes.byref(c_weights), float(eps), p, ws.data_ptr(),
                                  ws.numel(), _stream_ptr(z.device)), "fpb_pair_block")
    return (z, ws) if return_workspace else z


SINGLE_WEIGHTS = ("ln_a_w", "ln_a_b", "w_q", "b_q", "w_k", "w_v", "w_g", "w_o", "ln_z_w",
                  "ln_z_b", "w_z", "tr_ln_w", "tr_ln_b", "tr_w_a", "tr_w_b", "tr_w_out")


def single_block_workspace(n: int, rows: int, device) -> torch.Tensor:
    nbytes = _lib.load().fpb_single_block_workspace_size(n, rows, 384)
    if nbytes == 0:
        raise RuntimeError(f"unsupported single block size n={n} rows={rows}")
    return workspace(nbytes, device)


def single_block(s: torch.Tensor, z_loc: torch.Tensor, mask, c_weights, *, r0: int = 0,
                 precision="strict", eps: float = 1e-5, workspace=None,
                 return_workspace: bool = False):
    """Single stack of one Pairformer block in place on rows ``[r0, r0 +
    rows)`` of ``s`` ``[n, 384]``: ``s += AttentionPairBias(s, z)``, then
    ``s += Transition(s)``.

    ``z_loc`` holds the pair rows of those queries (``[rows, n, 128]``; the
    whole ``z`` when unsharded), ``mask`` is the full ``[n, n]`` pair mask or
    None, ``c_weights`` a ``modules.SingleBlockWeights`` struct. FP32 in both
    precision modes.
    """
    _require_cuda(s, z_loc, mask)
    if s.dtype != torch.float32 or s.ndim != 2 or s.shape[1] != 384:
        raise RuntimeError("single_block takes a float32 [n, 384] single tensor")
    n = s.shape[0]
    if z_loc.dtype != torch.float32 or z_loc.ndim != 3 or z_loc.shape[1:] != (n, 128):
        raise RuntimeError("z_loc must be a float32 [rows, n, 128] tensor")
    rows = z_loc.shape[0]
    for t, name in ((s, "s"), (z_loc, "z_loc")):
        if not t.is_contiguous() or t.data_ptr() % 16:
            raise RuntimeError(f"single_block needs a contiguous, 16-byte aligned {name}")
    if mask is not None:
        if tuple(mask.shape) != (n, n) or mask.dtype != torch.float32 or not mask.is_contiguous():
            raise RuntimeError("mask must be a contiguous float32 [n, n] tensor")
    lib = _lib.load()
    p = precision_code(precision)
    ws = workspace if workspace is not None else single_block_workspace(n, rows, s.device)
    _lib.check(lib.fpb_single_block(s.data_ptr(), z_loc.data_ptr(),
                                    0 if mask is None else mask.data_ptr(), n, rows, int(r0),
                                    384, ctypes.byref(c_weights), float(eps), p, ws.data_ptr(),
                                    ws.numel(), _stream_ptr(s.device)), "fpb_single_block")
    return (s, ws) if return_workspace else s


def triangle_contract(left: torch.Tensor, right: torch.Tensor, *, outgoing: bool,
                      precision="strict", return_workspace: bool = False):
    """ESMFold2's triangle contraction on channels-last ``[n, n, C]`` (or
    ``[1, n, n, C]``) FP32 tensors: outgoing ``x_ijc = sum_k l_ikc r_jkc``,
    incoming ``x_ijc = sum_k l_kic r_kjc``. Returns a new tensor shaped like
    ``left``."""
    _require_cuda(left, right)
    if left.shape != right.shape or left.dtype != torch.float32 or right.dtype != torch.float32:
        raise RuntimeError("triangle_contract takes two float32 tensors of one shape")
    shape = tuple(left.shape)
    if len(shape) == 4 and shape[0] == 1:
        shape3 = shape[1:]
    elif len(shape) == 3:
        shape3 = shape
    else:
        raise RuntimeError("triangle_contract takes [n, n, C] or [1, n, n, C]")
    n, n2, c = shape3
    if n != n2 or c % 32:
        raise RuntimeError("triangle_contract needs a square pair tensor and C % 32 == 0")
    left, right = left.contiguous(), right.contiguous()
    lib = _lib.load()
    p = precision_code(precision)
    out = torch.empty_like(left)
    ws = workspace(lib.fpb_triangle_contract_workspace_size(n, c, p), left.device)
    _lib.check(lib.fpb_triangle_contract(left.data_ptr(), right.data_ptr(), out.data_ptr(), n, c,
                                         int(bool(outgoing)), p, ws.data_ptr(), ws.numel(),
                                         _stream_ptr(left.device)), "fpb_triangle_contract")
    return (out, ws) if return_workspace else out


def timing_enable(on: bool = True) -> None:
    _lib.load().fpb_timing_enable(int(bool(on)))


def timing_collect() -> dict:
    """Per-kernel launches and total device milliseconds since timing_enable."""
    import json
    buf = ctypes.create_string_buffer(1 << 16)
    _lib.check(_lib.load().fpb_timing_collect(buf, len(buf)), "fpb_timing_collect")
    return json.loads(buf.value.decode())
