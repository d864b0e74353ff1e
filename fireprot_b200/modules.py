"""Pair-stack modules with the attribute surface of the Protenix modules the
reference hooks, computing on the B200 kernels.

Attribute names follow the upstream classes that
``python/fireprot/backends/amd/triangle_multiplication.py:284-293``,
``qkv_projection.py:36-49``, ``attention_gate.py:20-24`` and
``transition_projection.py:27-38`` inspect, so weights can be copied
one-to-one from a Protenix/OpenFold3 checkpoint (``load_from``). All
linears are ``torch.nn.Linear`` ([out, in] layout); the attention gate and
output linears carry biases as upstream ``Attention`` does.

These modules are inference-only: ``forward`` runs under ``torch.no_grad``
semantics and updates ``z`` in place (the reference's ``inplace_safe``
contract, ``test_packed_triangle.py:105``).
"""
from __future__ import annotations

import ctypes
import math

import torch
from torch import nn

from . import _lib, ops


def _linear(c_in, c_out, bias=False):
    return nn.Linear(c_in, c_out, bias=bias)


def _init_normal_(module: nn.Module, gen: torch.Generator) -> None:
    """N(0, 1/fan_in) weights, LayerNorm gamma=1/beta=0, zero biases."""
    for m in module.modules():
        if isinstance(m, nn.Linear):
            w = torch.randn(m.weight.shape, generator=gen) / math.sqrt(m.weight.shape[1])
            m.weight.data.copy_(w)
            if m.bias is not None:
                m.bias.data.zero_()
        elif isinstance(m, nn.LayerNorm):
            m.weight.data.fill_(1.0)
            m.bias.data.zero_()


class TriangleMultiplicativeUpdate(nn.Module):
    """Protenix ``TriangleMultiplicativeUpdate`` (bias-free linears)."""

    def __init__(self, c_z: int = 128, c_hidden: int = 128, _outgoing: bool = True):
        super().__init__()
        self.c_z, self.c_hidden, self._outgoing = c_z, c_hidden, _outgoing
        self.linear_a_p = _linear(c_z, c_hidden)
        self.linear_a_g = _linear(c_z, c_hidden)
        self.linear_b_p = _linear(c_z, c_hidden)
        self.linear_b_g = _linear(c_z, c_hidden)
        self.linear_g = _linear(c_z, c_z)
        self.linear_z = _linear(c_hidden, c_z)
        self.layer_norm_in = nn.LayerNorm(c_z)
        self.layer_norm_out = nn.LayerNorm(c_hidden)

    def weight_dict(self):
        return dict(ln_in_w=self.layer_norm_in.weight, ln_in_b=self.layer_norm_in.bias,
                    w_a_p=self.linear_a_p.weight, w_a_g=self.linear_a_g.weight,
                    w_b_p=self.linear_b_p.weight, w_b_g=self.linear_b_g.weight,
                    w_g=self.linear_g.weight, ln_out_w=self.layer_norm_out.weight,
                    ln_out_b=self.layer_norm_out.bias, w_z=self.linear_z.weight)

    @torch.no_grad()
    def forward(self, z, mask=None, *, add: bool = True, precision="strict"):
        return ops.trimul(z, mask, self.weight_dict(), outgoing=self._outgoing, add=add,
                          precision=precision, eps=self.layer_norm_in.eps)


class TriangleAttention(nn.Module):
    """Protenix ``TriangleAttention`` (``layer_norm``, bias projection
    ``linear``, and the ``mha`` q/k/v/g/o linears). ``starting=False`` is the
    ending node computed on the transposed pair tensor without a copy."""

    def __init__(self, c_in: int = 128, c_hidden: int = 32, no_heads: int = 4,
                 starting: bool = True, inf: float = 1e9):
        super().__init__()
        self.c_in, self.c_hidden, self.no_heads = c_in, c_hidden, no_heads
        self.starting, self.inf = starting, inf
        self.layer_norm = nn.LayerNorm(c_in)
        self.linear = _linear(c_in, no_heads)
        self.mha = nn.Module()
        self.mha.no_heads, self.mha.c_hidden = no_heads, c_hidden
        hd = c_hidden * no_heads
        self.mha.linear_q = _linear(c_in, hd)
        self.mha.linear_k = _linear(c_in, hd)
        self.mha.linear_v = _linear(c_in, hd)
        self.mha.linear_g = _linear(c_in, hd, bias=True)
        self.mha.linear_o = _linear(hd, c_in, bias=True)

    def weight_dict(self):
        m = self.mha
        return dict(ln_w=self.layer_norm.weight, ln_b=self.layer_norm.bias,
                    w_q=m.linear_q.weight, w_k=m.linear_k.weight, w_v=m.linear_v.weight,
                    w_bias=self.linear.weight, w_g=m.linear_g.weight, b_g=m.linear_g.bias,
                    w_o=m.linear_o.weight, b_o=m.linear_o.bias)

    @torch.no_grad()
    def forward(self, z, mask=None, *, precision="strict"):
        if self.inf != 1e9 or self.no_heads != 4 or self.c_hidden != 32:
            raise RuntimeError("the B200 kernel implements H=4, d=32, inf=1e9")
        return ops.triattn(z, mask, self.weight_dict(), starting=self.starting,
                           precision=precision, eps=self.layer_norm.eps)


class Transition(nn.Module):
    """Protenix pair ``Transition`` (SwiGLU, bias-free)."""

    def __init__(self, c_in: int = 128, n: int = 4):
        super().__init__()
        self.c_in, self.n = c_in, n
        self.layernorm1 = nn.LayerNorm(c_in)
        self.linear_no_bias_a = _linear(c_in, n * c_in)
        self.linear_no_bias_b = _linear(c_in, n * c_in)
        self.linear_no_bias = _linear(n * c_in, c_in)

    def weight_dict(self):
        return dict(ln_w=self.layernorm1.weight, ln_b=self.layernorm1.bias,
                    w_a=self.linear_no_bias_a.weight, w_b=self.linear_no_bias_b.weight,
                    w_out=self.linear_no_bias.weight)

    @torch.no_grad()
    def forward(self, z, *, precision="strict"):
        return ops.transition(z, self.weight_dict(), precision=precision,
                              eps=self.layernorm1.eps)


class _TriMulW(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in (
        "ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p", "w_b_g", "w_g", "ln_out_w", "ln_out_b",
        "w_z")]


class _TriAttnW(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in ops.TRIATTN_WEIGHTS]


class _TransW(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in ("ln_w", "ln_b", "w_a", "w_b", "w_out")]


class PairBlockWeights(ctypes.Structure):
    """Mirror of ``fpb_pair_block_weights`` (include/fireprot_b200.h)."""
    _fields_ = [("tri_mul_out", _TriMulW), ("tri_mul_in", _TriMulW),
                ("tri_att_start", _TriAttnW), ("tri_att_end", _TriAttnW),
                ("transition", _TransW)]


def _fill(struct, weights: dict, keep: list):
    for name, _ in struct._fields_:
        t = weights.get(name)
        if t is None:
            setattr(struct, name, None)
            continue
        if not t.is_cuda or t.dtype != torch.float32:
            raise RuntimeError(f"weight {name} must be a CUDA float32 tensor")
        t = t.contiguous()
        keep.append(t)
        setattr(struct, name, t.data_ptr())


class PairformerPairBlock(nn.Module):
    """Pair stack of one Pairformer block (AF3 Algorithm 17 order):
    TriMul out, TriMul in, TriAttn start, TriAttn end, transition."""

    def __init__(self, c_z: int = 128):
        super().__init__()
        self.tri_mul_out = TriangleMultiplicativeUpdate(c_z, c_z, True)
        self.tri_mul_in = TriangleMultiplicativeUpdate(c_z, c_z, False)
        self.tri_att_start = TriangleAttention(c_z, 32, 4, starting=True)
        self.tri_att_end = TriangleAttention(c_z, 32, 4, starting=False)
        self.pair_transition = Transition(c_z, 4)
        self._packed = None

    def init_random_(self, seed: int = 1) -> "PairformerPairBlock":
        _init_normal_(self, torch.Generator().manual_seed(seed))
        self._packed = None
        return self

    def c_weights(self):
        """ctypes weight struct (cached until the parameters change)."""
        key = tuple((p.data_ptr(), p._version) for p in self.parameters())
        if self._packed is None or self._packed[0] != key:
            keep: list = []
            w = PairBlockWeights()
            _fill(w.tri_mul_out, self.tri_mul_out.weight_dict(), keep)
            _fill(w.tri_mul_in, self.tri_mul_in.weight_dict(), keep)
            _fill(w.tri_att_start, self.tri_att_start.weight_dict(), keep)
            _fill(w.tri_att_end, self.tri_att_end.weight_dict(), keep)
            _fill(w.transition, self.pair_transition.weight_dict(), keep)
            self._packed = (key, w, keep)
        return self._packed[1]

    @torch.no_grad()
    def forward(self, z, mask=None, *, precision="strict", workspace=None):
        return ops.pair_block(z, mask, self.c_weights(), precision=precision,
                              workspace=workspace)


# --------------------------------------------------------------------------
# single stack
# --------------------------------------------------------------------------
class _GatedAttention(nn.Module):
    """The projections of upstream ``Attention`` as AttentionPairBias builds
    it (q with bias; k, v, gate and output bias-free)."""

    def __init__(self, c: int = 384, heads: int = 16):
        super().__init__()
        self.num_heads, self.c_hidden = heads, c // heads
        self.linear_q = _linear(c, c, bias=True)
        self.linear_k = _linear(c, c)
        self.linear_v = _linear(c, c)
        self.linear_g = _linear(c, c)
        self.linear_o = _linear(c, c)


class AttentionPairBias(nn.Module):
    """Protenix ``AttentionPairBias`` without conditioning (``has_s=False``):
    LayerNorm of s, gated multi-head attention over all tokens with one pair
    bias per head from ``linear_nobias_z(layernorm_z(z))``."""

    def __init__(self, c_a: int = 384, c_z: int = 128, n_heads: int = 16):
        super().__init__()
        self.n_heads = n_heads
        self.layernorm_a = nn.LayerNorm(c_a)
        self.attention = _GatedAttention(c_a, n_heads)
        self.layernorm_z = nn.LayerNorm(c_z)
        self.linear_nobias_z = _linear(c_z, n_heads)

    def weight_dict(self):
        at = self.attention
        return dict(ln_a_w=self.layernorm_a.weight, ln_a_b=self.layernorm_a.bias,
                    w_q=at.linear_q.weight, b_q=at.linear_q.bias, w_k=at.linear_k.weight,
                    w_v=at.linear_v.weight, w_g=at.linear_g.weight, w_o=at.linear_o.weight,
                    ln_z_w=self.layernorm_z.weight, ln_z_b=self.layernorm_z.bias,
                    w_z=self.linear_nobias_z.weight)


class SingleBlockWeights(ctypes.Structure):
    """Mirror of ``fpb_single_block_weights`` (include/fireprot_b200.h)."""
    _fields_ = [(k, ctypes.c_void_p) for k in ops.SINGLE_WEIGHTS]


class PairformerSingleBlock(nn.Module):
    """Single stack of one Pairformer block (AF3 Algorithm 17, lines 6-7):
    ``s += attention_pair_bias(s, z)``, ``s += single_transition(s)``;
    c_s = 384, 16 heads of 24."""

    def __init__(self, c_s: int = 384, c_z: int = 128, n_heads: int = 16):
        super().__init__()
        if c_s != 384 or c_z != 128 or n_heads != 16:
            raise RuntimeError("the B200 kernels implement c_s=384, c_z=128, 16 heads")
        self.attention_pair_bias = AttentionPairBias(c_s, c_z, n_heads)
        self.single_transition = Transition(c_s, 4)
        self._packed = None

    def init_random_(self, seed: int = 1) -> "PairformerSingleBlock":
        _init_normal_(self, torch.Generator().manual_seed(seed))
        self._packed = None
        return self

    def weight_dict(self):
        w = dict(self.attention_pair_bias.weight_dict())
        t = self.single_transition.weight_dict()
        w.update(tr_ln_w=t["ln_w"], tr_ln_b=t["ln_b"], tr_w_a=t["w_a"], tr_w_b=t["w_b"],
                 tr_w_out=t["w_out"])
        return w

    def c_weights(self):
        """ctypes weight struct (cached until the parameters change)."""
        key = tuple((p.data_ptr(), p._version) for p in self.parameters())
        if self._packed is None or self._packed[0] != key:
            keep: list = []
            w = SingleBlockWeights()
            _fill(w, self.weight_dict(), keep)
            self._packed = (key, w, keep)
        return self._packed[1]

    @torch.no_grad()
    def forward(self, s, z, mask=None, *, precision="strict", workspace=None):
        return ops.single_block(s, z, mask, self.c_weights(), precision=precision,
                                eps=self.single_transition.layernorm1.eps, workspace=workspace)


class PairformerBlock(nn.Module):
    """One whole Pairformer block: the pair stack on z, then the single stack
    on s reading the updated z (Protenix ``PairformerBlock`` order)."""

    def __init__(self, c_z: int = 128, c_s: int = 384, n_heads: int = 16):
        super().__init__()
        self.pair = PairformerPairBlock(c_z)
        self.single = PairformerSingleBlock(c_s, c_z, n_heads)

    def init_random_(self, seed: int = 1) -> "PairformerBlock":
        self.pair.init_random_(seed)
        self.single.init_random_(seed + 1000)
        return self

    @torch.no_grad()
    def forward(self, s, z, mask=None, *, precision="strict", workspace=None,
                single_workspace=None):
        self.pair(z, mask, precision=precision, workspace=workspace)
        self.single(s, z, mask, precision=precision, workspace=single_workspace)
        return s, z

    OPERATORS = ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end",
                 "pair_transition", "single")

    @torch.no_grad()
    def forward_by_operator(self, s, z, mask=None, *, precision="strict"):
        """The same block one operator at a time, for inspection: yields
        ``(name, tensor)`` after each operator has updated ``z`` (or, for the
        final ``"single"``, ``s``) in place, in ``OPERATORS`` order, with the
        stream synchronised. Same kernels as ``forward``; each operator gets
        its own workspace and its device status is checked."""
        pair = self.pair
        for name in self.OPERATORS[:5]:
            mod = getattr(pair, name)
            if name == "pair_transition":
                _, ws = ops.transition(z, mod.weight_dict(), precision=precision,
                                       return_workspace=True)
            elif name.startswith("tri_mul"):
                _, ws = ops.trimul(z, mask, mod.weight_dict(), outgoing=mod._outgoing,
                                   precision=precision, return_workspace=True)
            else:
                _, ws = ops.triattn(z, mask, mod.weight_dict(), starting=mod.starting,
                                    precision=precision, return_workspace=True)
            if ops.workspace_status(ws) != 0:
                raise RuntimeError(f"{name}: device status {ops.workspace_status(ws)}")
            yield name, z
        _, ws = ops.single_block(s, z, mask, self.single.c_weights(), precision=precision,
                                 return_workspace=True)
        if ops.workspace_status(ws) != 0:
            raise RuntimeError(f"single: device status {ops.workspace_status(ws)}")
        yield "single", s
