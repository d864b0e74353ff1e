"""CPU restatement of the reference's native Pairformer pair-path math.

TEST INFRASTRUCTURE ONLY. This module is the parity checker for the CUDA
backend in ``fireprot_b200``. It is imported by ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``; the
product path never imports or calls it.

Parity pinning: the golden fixtures in ``tests/golden`` are produced by running
the reference's own Python functions (``adapters/atlasfold/runtime.py``
``triangle_attention`` / ``triangle_multiplication``,
``backends/amd/triangle_multiplication.py`` ``_short_sequence_hip_fused``,
``backends/amd/recycle.py`` ``_hip_transition`` and
``backends/amd/triangle_attention.py`` ``_efficient_sdpa``) with torch
stand-ins for their HIP elementwise helpers; ``tests/test_oracle_golden.py``
checks this restatement against them.

All arithmetic is torch on the CPU in the dtype of the inputs (float32 for
parity, float64 for a second opinion). Layouts follow the reference: the pair
tensor ``z`` is ``[N, N, c_z]`` channels-last, masks are ``[N, N]`` with 1 =
valid.

Reference citations (paths inside the reference project):
- LayerNorm eps 1e-5: ``python/fireprot/backends/amd/recycle.py:101``.
- Triangle multiplication order (mask/gate/LN_out/linear_z/residual):
  ``python/fireprot/backends/amd/triangle_multiplication.py:162-193`` and the
  contraction directions of ``python/fireprot/backends/amd/lt_bmm.py:85``.
- Triangle attention (LN -> q/k/v -> bias -> mask -> softmax -> gate -> out):
  ``python/fireprot/adapters/atlasfold/runtime.py:32-71``; Q pre-scaled by
  1/sqrt(d) (``kernels/amd/fireprot_amd_ops.cu:915``); mask bias
  ``1e9 * (mask - 1)`` (``patches/protenix/0005-...patch:35-38``).
- Ending node = starting-node math on the transposed pair tensor, output
  transposed back (``patches/protenix/0006-...patch:22,34``).
- Pair transition ``W_out(silu(LN(z) W_a^T) * (LN(z) W_b^T))``:
  ``python/fireprot/backends/amd/recycle.py:203-227``.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import torch

LN_EPS = 1e-5
MASK_INF = 1e9


# --------------------------------------------------------------------------
# parameters (names mirror the Protenix modules the reference hooks)
# --------------------------------------------------------------------------
@dataclasses.dataclass
class TriMulParams:
    """Weights of one ``TriangleMultiplicativeUpdate`` (all linears bias-free).

    Mirrors ``linear_a_p/linear_a_g/linear_b_p/linear_b_g/linear_g/linear_z``
    and ``layer_norm_in/layer_norm_out`` checked at
    ``python/fireprot/backends/amd/triangle_multiplication.py:284-293``.
    """
    ln_in_w: torch.Tensor
    ln_in_b: torch.Tensor
    w_a_p: torch.Tensor  # [c_hidden, c_z]
    w_a_g: torch.Tensor
    w_b_p: torch.Tensor
    w_b_g: torch.Tensor
    w_g: torch.Tensor    # [c_z, c_z]
    ln_out_w: torch.Tensor
    ln_out_b: torch.Tensor
    w_z: torch.Tensor    # [c_z, c_hidden]


@dataclasses.dataclass
class TriAttnParams:
    """Weights of one ``TriangleAttention`` (``layer_norm``, ``linear`` for the
    pair bias and the ``mha`` q/k/v/g/o linears).

    ``b_g`` / ``b_o`` are the optional gating / output biases of the
    upstream ``Attention`` module (``attention_gate.py:28-56`` accepts both).
    """
    ln_w: torch.Tensor
    ln_b: torch.Tensor
    w_q: torch.Tensor    # [H*d, c_z]
    w_k: torch.Tensor
    w_v: torch.Tensor
    w_bias: torch.Tensor  # [H, c_z]
    w_g: torch.Tensor    # [H*d, c_z]
    w_o: torch.Tensor    # [c_z, H*d]
    heads: int
    head_dim: int
    b_g: Optional[torch.Tensor] = None
    b_o: Optional[torch.Tensor] = None


@dataclasses.dataclass
class TransitionParams:
    """Weights of the pair ``Transition`` (``layernorm1``, ``linear_no_bias_a``,
    ``linear_no_bias_b``, ``linear_no_bias``; ``transition_projection.py:27-38``)."""
    ln_w: torch.Tensor
    ln_b: torch.Tensor
    w_a: torch.Tensor    # [n*c, c]
    w_b: torch.Tensor    # [n*c, c]
    w_out: torch.Tensor  # [c, n*c]


@dataclasses.dataclass
class PairBlockParams:
    tri_mul_out: TriMulParams
    tri_mul_in: TriMulParams
    tri_att_start: TriAttnParams
    tri_att_end: TriAttnParams
    transition: TransitionParams


def _normal(gen, shape, std, dtype):
    return (torch.randn(*shape, generator=gen, dtype=torch.float32) * std).to(dtype)


def make_trimul_params(c_z=128, c_hidden=128, seed=1, dtype=torch.float32,
                       ln_affine_random=False) -> TriMulParams:
    """Seeded random-init weights ~ N(0, 1/fan_in)."""
    g = torch.Generator().manual_seed(seed)
    s_in, s_h = 1.0 / math.sqrt(c_z), 1.0 / math.sqrt(c_hidden)
    if ln_affine_random:
        ln = [1.0 + 0.1 * torch.randn(c_z, generator=g), 0.1 * torch.randn(c_z, generator=g),
              1.0 + 0.1 * torch.randn(c_hidden, generator=g), 0.1 * torch.randn(c_hidden, generator=g)]
    else:
        ln = [torch.ones(c_z), torch.zeros(c_z), torch.ones(c_hidden), torch.zeros(c_hidden)]
    return TriMulParams(
        ln_in_w=ln[0].to(dtype), ln_in_b=ln[1].to(dtype),
        w_a_p=_normal(g, (c_hidden, c_z), s_in, dtype),
        w_a_g=_normal(g, (c_hidden, c_z), s_in, dtype),
        w_b_p=_normal(g, (c_hidden, c_z), s_in, dtype),
        w_b_g=_normal(g, (c_hidden, c_z), s_in, dtype),
        w_g=_normal(g, (c_z, c_z), s_in, dtype),
        ln_out_w=ln[2].to(dtype), ln_out_b=ln[3].to(dtype),
        w_z=_normal(g, (c_z, c_hidden), s_h, dtype),
    )


def make_triattn_params(c_z=128, heads=4, head_dim=32, seed=1, dtype=torch.float32,
                        with_biases=False, ln_affine_random=False) -> TriAttnParams:
    """Seeded random-init weights. BASELINE config 1 uses N(0, 1/128) for
    W_q/k/v/g, LN gamma=1 / beta=0 and no gate/output bias."""
    g = torch.Generator().manual_seed(seed)
    hd = heads * head_dim
    s_in, s_h = 1.0 / math.sqrt(c_z), 1.0 / math.sqrt(hd)
    if ln_affine_random:
        ln_w = 1.0 + 0.1 * torch.randn(c_z, generator=g)
        ln_b = 0.1 * torch.randn(c_z, generator=g)
    else:
        ln_w, ln_b = torch.ones(c_z), torch.zeros(c_z)
    p = TriAttnParams(
        ln_w=ln_w.to(dtype), ln_b=ln_b.to(dtype),
        w_q=_normal(g, (hd, c_z), s_in, dtype),
        w_k=_normal(g, (hd, c_z), s_in, dtype),
        w_v=_normal(g, (hd, c_z), s_in, dtype),
        w_bias=_normal(g, (heads, c_z), s_in, dtype),
        w_g=_normal(g, (hd, c_z), s_in, dtype),
        w_o=_normal(g, (c_z, hd), s_h, dtype),
        heads=heads, head_dim=head_dim,
    )
    if with_biases:
        p.b_g = _normal(g, (hd,), 1.0, dtype)
        p.b_o = _normal(g, (c_z,), 0.1, dtype)
    return p


def make_transition_params(c=128, n=4, seed=1, dtype=torch.float32,
                           ln_affine_random=False) -> TransitionParams:
    g = torch.Generator().manual_seed(seed)
    if ln_affine_random:
        ln_w = 1.0 + 0.1 * torch.randn(c, generator=g)
        ln_b = 0.1 * torch.randn(c, generator=g)
    else:
        ln_w, ln_b = torch.ones(c), torch.zeros(c)
    return TransitionParams(
        ln_w=ln_w.to(dtype), ln_b=ln_b.to(dtype),
        w_a=_normal(g, (n * c, c), 1.0 / math.sqrt(c), dtype),
        w_b=_normal(g, (n * c, c), 1.0 / math.sqrt(c), dtype),
        w_out=_normal(g, (c, n * c), 1.0 / math.sqrt(n * c), dtype),
    )


def make_block_params(c_z=128, seed=1, dtype=torch.float32) -> PairBlockParams:
    return PairBlockParams(
        tri_mul_out=make_trimul_params(c_z, c_z, seed=seed, dtype=dtype),
        tri_mul_in=make_trimul_params(c_z, c_z, seed=seed + 1, dtype=dtype),
        tri_att_start=make_triattn_params(c_z, seed=seed + 2, dtype=dtype),
        tri_att_end=make_triattn_params(c_z, seed=seed + 3, dtype=dtype),
        transition=make_transition_params(c_z, seed=seed + 4, dtype=dtype),
    )


def make_pair(n, c=128, seed=0, dtype=torch.float32) -> torch.Tensor:
    """Seeded z ~ N(0, 1) of shape [n, n, c] (``torch.Generator().manual_seed``)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, n, c, generator=g, dtype=torch.float32).to(dtype)


def make_padding_mask(n, valid, dtype=torch.float32) -> torch.Tensor:
    """Pair mask of a padded sequence: rows and columns >= valid are 0."""
    v = torch.arange(n) < valid
    return (v[:, None] & v[None, :]).to(dtype)


# --------------------------------------------------------------------------
# primitives
# --------------------------------------------------------------------------
def layer_norm(x, w, b, eps=LN_EPS):
    """LayerNorm over the last dim (biased variance), as torch's native op."""
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


def attention_core(q, k, v, biases, empty_rows="nan"):
    """The upstream ``_attention``: ``softmax(q @ k^T + sum(biases)) @ v``.

    q, k, v: ``[*, H, Q, D]``; biases broadcast to ``[*, H, Q, K]`` and are
    added in list order (mask bias first). Q is pre-scaled by the caller.
    Returns ``[*, H, Q, D]`` (the reference's dispatch transposes it to
    ``[*, Q, H, D]``; ``triangle_attention.py:129``).

    ``empty_rows`` is the result of a query row whose every logit is -inf:
    ``"nan"`` as torch's softmax (upstream ``_attention``, and the OpenFold3
    kernel's zero-row-sum contract, ``fireprot_softmax_fp32.cpp:61-62``),
    ``"zero"`` as torch's ``scaled_dot_product_attention``, which the
    Protenix dispatch checks its kernels against (``triangle_attention.py:
    83-129``; ``tests/operators/test_ck_attention.py:69-81``).
    """
    a = torch.matmul(q, k.transpose(-1, -2))
    for b in biases:
        a = a + b
    empty = None
    if empty_rows == "zero":
        empty = torch.isneginf(a.amax(dim=-1, keepdim=True))
    elif empty_rows != "nan":
        raise ValueError(empty_rows)
    a = torch.softmax(a, dim=-1)
    out = torch.matmul(a, v)
    if empty is not None:
        out = out.masked_fill(empty, 0.0)
    return out


# --------------------------------------------------------------------------
# pair operators
# --------------------------------------------------------------------------
def triangle_multiplication(z, mask, p: TriMulParams, *, outgoing: bool, add: bool = True):
    """Protenix ``TriangleMultiplicativeUpdate`` inference semantics.

    ``a = mask * sigmoid(LN(z) W_a_g^T) * (LN(z) W_a_p^T)`` (b likewise),
    outgoing ``x_ij = sum_k a_ik b_jk``, incoming ``x_ij = sum_k a_ki b_kj``,
    ``delta = sigmoid(LN(z) W_g^T) * (LN_out(x) W_z^T)``; the gate uses the
    unmasked LN(z) (``triangle_multiplication.py:162-193``). Returns ``z +
    delta`` when ``add`` else ``delta`` (``fireprot_amd_ops.cu:589-601``).
    """
    zn = layer_norm(z, p.ln_in_w, p.ln_in_b)
    a = torch.sigmoid(zn @ p.w_a_g.T) * (zn @ p.w_a_p.T)
    b = torch.sigmoid(zn @ p.w_b_g.T) * (zn @ p.w_b_p.T)
    if mask is not None:
        a = a * mask[..., None]
        b = b * mask[..., None]
    a_cf = a.permute(2, 0, 1)  # [c, N, N]
    b_cf = b.permute(2, 0, 1)
    if outgoing:
        x = torch.matmul(a_cf, b_cf.transpose(-1, -2))  # sum_k a[c,i,k] b[c,j,k]
    else:
        x = torch.matmul(a_cf.transpose(-1, -2), b_cf)  # sum_k a[c,k,i] b[c,k,j]
    x = x.permute(1, 2, 0)
    x = layer_norm(x, p.ln_out_w, p.ln_out_b)
    x = x @ p.w_z.T
    g = torch.sigmoid(zn @ p.w_g.T)
    delta = g * x
    return z + delta if add else delta


def triangle_attention(z, mask, p: TriAttnParams, *, starting: bool = True, chunk: int = 64):
    """Triangle attention update ``delta`` (without the residual add).

    Starting node: for row i, ``o_ij = sum_k softmax_k(q_ij.k_ik / sqrt(d) +
    b^h_jk + 1e9 (mask_ik - 1)) v_ik``; ``delta_ij = W_o(g_ij * o_ij) + b_o``
    with ``g = sigmoid(LN(z) W_g^T + b_g)`` and ``b^h = LN(z) W_bias^T``.
    Ending node: the same on ``z^T`` (and ``mask^T``), result transposed back.
    Follows ``adapters/atlasfold/runtime.py:32-71``; rows are processed in
    chunks of ``chunk`` to bound the ``[chunk, H, N, N]`` score buffer.
    """
    x = z if starting else z.transpose(0, 1)
    m = None if mask is None else (mask if starting else mask.transpose(0, 1))
    n = x.shape[0]
    H, d = p.heads, p.head_dim
    xn = layer_norm(x, p.ln_w, p.ln_b)
    scale = 1.0 / math.sqrt(d)
    q = (xn @ p.w_q.T).reshape(n, n, H, d).permute(0, 2, 1, 3) * scale  # [i,h,j,d]
    k = (xn @ p.w_k.T).reshape(n, n, H, d).permute(0, 2, 1, 3)
    v = (xn @ p.w_v.T).reshape(n, n, H, d).permute(0, 2, 1, 3)
    tri_bias = (xn @ p.w_bias.T).permute(2, 0, 1).unsqueeze(0)  # [1,h,j,k]
    gate = xn @ p.w_g.T
    if p.b_g is not None:
        gate = gate + p.b_g
    gate = torch.sigmoid(gate)
    outs = []
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        biases = []
        if m is not None:
            biases.append((MASK_INF * (m[s:e] - 1.0))[:, None, None, :])
        biases.append(tri_bias)
        o = attention_core(q[s:e], k[s:e], v[s:e], biases)  # [c,h,j,d]
        outs.append(o.permute(0, 2, 1, 3).reshape(e - s, n, H * d))
    o = torch.cat(outs, 0)
    out = (gate * o) @ p.w_o.T
    if p.b_o is not None:
        out = out + p.b_o
    return out if starting else out.transpose(0, 1)


def pair_transition(z, p: TransitionParams):
    """Pair transition update ``W_out(silu(LN(z) W_a^T) * (LN(z) W_b^T))``."""
    xn = layer_norm(z, p.ln_w, p.ln_b)
    return (torch.nn.functional.silu(xn @ p.w_a.T) * (xn @ p.w_b.T)) @ p.w_out.T


def pair_block(z, mask, p: PairBlockParams, *, attn_chunk: int = 64):
    """Pair stack of one Pairformer block (AF3 Algorithm 17 order):
    TriMul out, TriMul in, TriAttn start, TriAttn end, transition; each adds
    its update to z (``patches/protenix/0006-...patch:14-37``)."""
    z = triangle_multiplication(z, mask, p.tri_mul_out, outgoing=True, add=True)
    z = triangle_multiplication(z, mask, p.tri_mul_in, outgoing=False, add=True)
    z = z + triangle_attention(z, mask, p.tri_att_start, starting=True, chunk=attn_chunk)
    z = z + triangle_attention(z, mask, p.tri_att_end, starting=False, chunk=attn_chunk)
    z = z + pair_transition(z, p.transition)
    return z


# --------------------------------------------------------------------------
# row-sampled forms (full-size parity: the same math on a few rows)
# --------------------------------------------------------------------------
# Each function returns selected rows (or, for the ending node, columns) of
# the corresponding full operator above, computing only what those rows
# depend on: the terms that couple rows (TriMul's b over every pair, the
# pair bias of TriAttn over every pair) in full, the rest for the selected
# rows. Used to check CUDA results at sizes where the full CPU restatement
# would take minutes (N = 1000, 1536, 3072).
def _idx(rows):
    return torch.as_tensor(rows, dtype=torch.long)


def trimul_rows(z, mask, p: TriMulParams, rows, *, outgoing: bool, add: bool = True):
    """Rows ``rows`` of ``triangle_multiplication(z, mask, p, ...)``
    (``[len(rows), N, c_z]``). Outgoing row i needs a[i, :] and all of b;
    incoming row i needs a[:, i] and all of b."""
    r = _idx(rows)
    zn = layer_norm(z, p.ln_in_w, p.ln_in_b)
    b = torch.sigmoid(zn @ p.w_b_g.T) * (zn @ p.w_b_p.T)
    if mask is not None:
        b = b * mask[..., None]
    za = zn[r] if outgoing else zn[:, r]          # [r, k, c] or [k, r, c]
    a = torch.sigmoid(za @ p.w_a_g.T) * (za @ p.w_a_p.T)
    if mask is not None:
        a = a * (mask[r] if outgoing else mask[:, r])[..., None]
    a_cf = a.permute(2, 0, 1) if outgoing else a.permute(2, 1, 0)  # [c, r, k]
    b_cf = b.permute(2, 0, 1)                                      # [c, N, N]
    if outgoing:
        x = torch.matmul(a_cf, b_cf.transpose(-1, -2))  # sum_k a[c,i,k] b[c,j,k]
    else:
        x = torch.matmul(a_cf, b_cf)                    # sum_k a[c,k,i] b[c,k,j]
    x = layer_norm(x.permute(1, 2, 0), p.ln_out_w, p.ln_out_b) @ p.w_z.T
    delta = torch.sigmoid(zn[r] @ p.w_g.T) * x
    return z[r] + delta if add else delta


def triattn_lines(z, mask, p: TriAttnParams, lines, *, starting: bool = True, chunk: int = 8):
    """Lines of the triangle attention update (no residual), as
    ``[len(lines), N, c_z]``: starting node, rows ``delta[l, :]``; ending
    node, columns ``delta[:, l]`` (row l of the starting-node form on z^T).
    Each line needs its own pair line of z and the pair bias of every pair."""
    x = z if starting else z.transpose(0, 1)
    m = None if mask is None else (mask if starting else mask.transpose(0, 1))
    r = _idx(lines)
    n = x.shape[0]
    H, d = p.heads, p.head_dim
    tri_bias = (layer_norm(x, p.ln_w, p.ln_b) @ p.w_bias.T).permute(2, 0, 1).unsqueeze(0)
    outs = []
    for s in range(0, len(r), chunk):
        rr = r[s:s + chunk]
        xn = layer_norm(x[rr], p.ln_w, p.ln_b)                         # [c, N, C]
        q = (xn @ p.w_q.T).reshape(len(rr), n, H, d).permute(0, 2, 1, 3) / math.sqrt(d)
        k = (xn @ p.w_k.T).reshape(len(rr), n, H, d).permute(0, 2, 1, 3)
        v = (xn @ p.w_v.T).reshape(len(rr), n, H, d).permute(0, 2, 1, 3)
        biases = []
        if m is not None:
            biases.append((MASK_INF * (m[rr] - 1.0))[:, None, None, :])
        biases.append(tri_bias)
        o = attention_core(q, k, v, biases).permute(0, 2, 1, 3).reshape(len(rr), n, H * d)
        gate = xn @ p.w_g.T
        if p.b_g is not None:
            gate = gate + p.b_g
        out = (torch.sigmoid(gate) * o) @ p.w_o.T
        if p.b_o is not None:
            out = out + p.b_o
        outs.append(out)
    return torch.cat(outs, 0)


def transition_rows(z, p: TransitionParams, rows):
    """Rows of ``z + pair_transition(z, p)`` (the transition is row-local)."""
    zr = z[_idx(rows)]
    return zr + pair_transition(zr, p)


def single_block_rows(s, z, mask, p: "SingleBlockParams", rows):
    """Rows of ``single_block(s, z, mask, p)``: query row i needs its own
    pair row z[i] (the pair bias of its keys) and every row of s (keys and
    values); the transition is row-local."""
    r = _idx(rows)
    n = s.shape[0]
    h, d = p.heads, p.head_dim
    a = layer_norm(s, p.ln_a_w, p.ln_a_b)
    q = ((a[r] @ p.w_q.T + p.b_q) / math.sqrt(d)).view(len(r), h, d).transpose(0, 1)
    k = (a @ p.w_k.T).view(n, h, d).transpose(0, 1)
    v = (a @ p.w_v.T).view(n, h, d).transpose(0, 1)
    bias = (layer_norm(z[r], p.ln_z_w, p.ln_z_b) @ p.w_z.T).permute(2, 0, 1)  # [H, r, N]
    biases = [bias]
    if mask is not None:
        biases = [(MASK_INF * (mask[r] - 1.0)).to(s.dtype)[None], bias]
    o = attention_core(q, k, v, biases).transpose(0, 1).reshape(len(r), h * d)
    s1 = s[r] + (torch.sigmoid(a[r] @ p.w_g.T) * o) @ p.w_o.T
    return s1 + pair_transition(s1, p.transition)


def sample_lines(n: int, count: int = 12, seed: int = 0, valid=None):
    """Sorted distinct line indices: the first and last line, the last valid
    line and the first padded one (when ``valid`` < n), and ``count`` seeded
    random others."""
    g = torch.Generator().manual_seed(seed)
    pick = {0, n - 1}
    if valid is not None and 0 < valid < n:
        pick |= {valid - 1, valid}
    extra = torch.randperm(n, generator=g)[:count].tolist()
    return sorted(pick | set(extra))


# --------------------------------------------------------------------------
# ESMFold2 triangle contraction (channels last, C = 256 upstream)
# --------------------------------------------------------------------------
def triangle_contract(left, right, *, outgoing: bool):
    """``python/fireprot/adapters/esmfold2/triangle.py:19-33``: outgoing
    ``x_ijc = sum_k l_ikc r_jkc``, incoming ``x_ijc = sum_k l_kic r_kjc`` on
    ``[..., n, n, C]`` tensors. Its loop over chunks of i only bounds memory
    (every output element is one dot product over k), so the restatement is
    one einsum per direction."""
    if outgoing:
        return torch.einsum("...ikc,...jkc->...ijc", left, right)
    return torch.einsum("...kic,...kjc->...ijc", left, right)


# --------------------------------------------------------------------------
# tolerance checks (north star: strict 1e-4, fast 1e-2, relative to the
# fp32 output scale max|ref|)
# --------------------------------------------------------------------------
STRICT_TOL = 1e-4
FAST_TOL = 1e-2


def rel_max_err(actual, expected):
    """max|actual - expected| / max|expected| (the output-scale relative error)."""
    a = actual.detach().to("cpu", torch.float64)
    e = expected.detach().to("cpu", torch.float64)
    scale = e.abs().max().item()
    return (a - e).abs().max().item() / (scale if scale > 0 else 1.0)


# --------------------------------------------------------------------------
# single stack of a Pairformer block (next-row scope beyond the pair path)
# --------------------------------------------------------------------------
# Parity unpinned: the reference runs this stack natively through upstream
# Protenix (commit bb3be993, not vendored; ``docs/openfold3-performance.md:68-74``
# times it as "Single attention with pair bias" and "Single transition"), so
# there is no reference function or golden vector to pin it to. The
# restatement follows the published AlphaFold 3 supplement: Algorithm 24
# (AttentionPairBias, without the conditioning signal) and Algorithm 11
# (Transition), with the Pairformer's order s += APB(s, z); s += T(s).
@dataclasses.dataclass
class SingleBlockParams:
    """Weights of the single stack: ``AttentionPairBias`` (LayerNorm of s,
    q with bias, bias-free k/v/gate/output, LayerNorm + bias-free linear of z
    to one bias per head) and the single ``Transition``."""
    heads: int
    head_dim: int
    ln_a_w: torch.Tensor
    ln_a_b: torch.Tensor
    w_q: torch.Tensor   # [H*d, c_s]
    b_q: torch.Tensor   # [H*d]
    w_k: torch.Tensor   # [H*d, c_s]
    w_v: torch.Tensor   # [H*d, c_s]
    w_g: torch.Tensor   # [H*d, c_s]
    w_o: torch.Tensor   # [c_s, H*d]
    ln_z_w: torch.Tensor
    ln_z_b: torch.Tensor
    w_z: torch.Tensor   # [H, c_z]
    transition: TransitionParams


def make_single_params(c_s=384, c_z=128, heads=16, head_dim=24, seed=1, dtype=torch.float32,
                       ln_affine_random=False) -> SingleBlockParams:
    """Seeded random-init weights ~ N(0, 1/fan_in); defaults are the
    Pairformer's single stack (c_s 384, 16 heads of 24)."""
    g = torch.Generator().manual_seed(seed)
    hd = heads * head_dim
    if ln_affine_random:
        ln = [1.0 + 0.1 * torch.randn(c_s, generator=g), 0.1 * torch.randn(c_s, generator=g),
              1.0 + 0.1 * torch.randn(c_z, generator=g), 0.1 * torch.randn(c_z, generator=g)]
    else:
        ln = [torch.ones(c_s), torch.zeros(c_s), torch.ones(c_z), torch.zeros(c_z)]
    s_s, s_h, s_z = 1.0 / math.sqrt(c_s), 1.0 / math.sqrt(hd), 1.0 / math.sqrt(c_z)
    return SingleBlockParams(
        heads=heads, head_dim=head_dim,
        ln_a_w=ln[0].to(dtype), ln_a_b=ln[1].to(dtype),
        w_q=_normal(g, (hd, c_s), s_s, dtype),
        b_q=_normal(g, (hd,), 0.1, dtype),
        w_k=_normal(g, (hd, c_s), s_s, dtype),
        w_v=_normal(g, (hd, c_s), s_s, dtype),
        w_g=_normal(g, (hd, c_s), s_s, dtype),
        w_o=_normal(g, (c_s, hd), s_h, dtype),
        ln_z_w=ln[2].to(dtype), ln_z_b=ln[3].to(dtype),
        w_z=_normal(g, (heads, c_z), s_z, dtype),
        transition=make_transition_params(c_s, seed=seed + 100, dtype=dtype,
                                          ln_affine_random=ln_affine_random),
    )


def make_single(n, c=384, seed=0, dtype=torch.float32) -> torch.Tensor:
    """Seeded s ~ N(0, 1) of shape [n, c]."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, c, generator=g, dtype=torch.float32).to(dtype)


def attention_pair_bias(s, z, mask, p: SingleBlockParams):
    """AlphaFold 3 Algorithm 24 without conditioning, returning the update:
    ``a = LN(s)``; ``q = (a W_q^T + b_q) / sqrt(d)``; ``k, v, g`` bias-free;
    ``b^h_ij = LN(z_ij) W_z^T + 1e9 (mask_ij - 1)``;
    ``out = (sigmoid(a W_g^T) * softmax_j(q k^T + b) v) W_o^T``."""
    n = s.shape[0]
    h, d = p.heads, p.head_dim
    a = layer_norm(s, p.ln_a_w, p.ln_a_b)
    q = ((a @ p.w_q.T + p.b_q) / math.sqrt(d)).view(n, h, d).transpose(0, 1)
    k = (a @ p.w_k.T).view(n, h, d).transpose(0, 1)
    v = (a @ p.w_v.T).view(n, h, d).transpose(0, 1)
    bias = (layer_norm(z, p.ln_z_w, p.ln_z_b) @ p.w_z.T).permute(2, 0, 1)  # [H, i, j]
    biases = [bias]
    if mask is not None:
        biases = [(MASK_INF * (mask - 1.0)).to(s.dtype)[None], bias]
    o = attention_core(q, k, v, biases).transpose(0, 1).reshape(n, h * d)
    return (torch.sigmoid(a @ p.w_g.T) * o) @ p.w_o.T


def single_block(s, z, mask, p: SingleBlockParams):
    """Single stack of one Pairformer block: ``s += APB(s, z)``, then
    ``s += Transition(s)`` (AlphaFold 3 Algorithm 17, lines 6-7)."""
    s = s + attention_pair_bias(s, z, mask, p)
    return s + pair_transition(s, p.transition)
