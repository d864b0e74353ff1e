"""Single stack of a Pairformer block on CPU: the oracle restatement
(AlphaFold 3 Algorithm 24 without conditioning + Algorithm 11; parity
unpinned, the reference runs this stack natively through upstream Protenix)
checked against an independent loop form and for the invariances the
padding mask promises, plus the host-side boundary of ``fpb_single_block``
(argument validation before any launch, struct layout shared with the
header)."""
from __future__ import annotations

import ctypes
import math
import re
from pathlib import Path

import pytest
import torch

from oracle import pairformer_oracle as O

ROOT = Path(__file__).resolve().parents[1]


def _loop_attention_pair_bias(s, z, mask, p):
    """Per-head, per-query restatement with explicit softmax sums."""
    n = s.shape[0]
    h, d = p.heads, p.head_dim
    a = O.layer_norm(s, p.ln_a_w, p.ln_a_b)
    zb = O.layer_norm(z, p.ln_z_w, p.ln_z_b)
    out = torch.zeros(n, h * d, dtype=s.dtype)
    for hh in range(h):
        sl = slice(hh * d, (hh + 1) * d)
        q = (a @ p.w_q[sl].T + p.b_q[sl]) / math.sqrt(d)
        k = a @ p.w_k[sl].T
        v = a @ p.w_v[sl].T
        for i in range(n):
            logits = k @ q[i] + zb[i] @ p.w_z[hh]
            if mask is not None:
                logits = logits + O.MASK_INF * (mask[i] - 1.0)
            w = torch.exp(logits - logits.max())
            out[i, sl] = (w[:, None] * v).sum(0) / w.sum()
    return (torch.sigmoid(a @ p.w_g.T) * out) @ p.w_o.T


@pytest.mark.parametrize("mask_kind", ["none", "padding"])
def test_oracle_matches_loop_form(mask_kind):
    n = 9
    p = O.make_single_params(seed=2, dtype=torch.float64, ln_affine_random=True)
    s = O.make_single(n, seed=1, dtype=torch.float64)
    z = O.make_pair(n, seed=2, dtype=torch.float64)
    mask = None if mask_kind == "none" else O.make_padding_mask(n, 6, dtype=torch.float64)
    ref = _loop_attention_pair_bias(s, z, mask, p)
    out = O.attention_pair_bias(s, z, mask, p)
    assert O.rel_max_err(out[:6], ref[:6]) <= 1e-12
    # fully masked query rows: logits near -1e9 keep ~1e-7 absolute precision
    assert O.rel_max_err(out, ref) <= 1e-6


def test_oracle_float32_tracks_float64():
    n = 48
    p64 = O.make_single_params(seed=4, dtype=torch.float64, ln_affine_random=True)
    p32 = O.make_single_params(seed=4, dtype=torch.float32, ln_affine_random=True)
    s = O.make_single(n, seed=3)
    z = O.make_pair(n, seed=4)
    mask = O.make_padding_mask(n, 40)
    r64 = O.single_block(s.double(), z.double(), mask.double(), p64)
    r32 = O.single_block(s, z, mask, p32)
    assert O.rel_max_err(r32[:40], r64[:40]) <= 1e-5
    # Fully masked query rows: in FP32 every logit rounds to exactly -1e9
    # (|q.k + b| < 32, half the spacing of FP32 there), so their softmax is
    # uniform, as in the reference's FP32 math; FP64 keeps the differences.
    a = O.layer_norm(s, p32.ln_a_w, p32.ln_a_b)
    v_mean = (a @ p32.w_v.T).mean(0)
    upd = (torch.sigmoid(a @ p32.w_g.T) * v_mean) @ p32.w_o.T
    s1 = s + upd
    uniform = s1 + O.pair_transition(s1, p32.transition)
    assert O.rel_max_err(r32[40:], uniform[40:]) <= 1e-5


def test_padding_tokens_do_not_reach_valid_rows():
    """With a padding mask, valid query rows ignore the padded tokens' s and z."""
    n, valid = 24, 17
    p = O.make_single_params(seed=5, dtype=torch.float64)
    s = O.make_single(n, seed=5, dtype=torch.float64)
    z = O.make_pair(n, seed=6, dtype=torch.float64)
    mask = O.make_padding_mask(n, valid, dtype=torch.float64)
    ref = O.single_block(s, z, mask, p)
    s2, z2 = s.clone(), z.clone()
    s2[valid:] = 100.0 * torch.randn(n - valid, s.shape[1], dtype=torch.float64)
    z2[:, valid:] = -50.0
    z2[valid:] = 7.0
    out = O.single_block(s2, z2, mask, p)
    assert torch.allclose(out[:valid], ref[:valid], rtol=0, atol=1e-12)


def test_header_struct_matches_binding():
    from fireprot_b200 import modules, ops
    text = (ROOT / "include" / "fireprot_b200.h").read_text()
    body = re.search(r"typedef struct \{([^}]*)\} fpb_single_block_weights;", text).group(1)
    names = re.findall(r"\*(\w+)", body)
    assert tuple(names) == ops.SINGLE_WEIGHTS
    assert [f for f, _ in modules.SingleBlockWeights._fields_] == list(ops.SINGLE_WEIGHTS)
    blk = modules.PairformerSingleBlock()
    assert tuple(blk.weight_dict()) == ops.SINGLE_WEIGHTS


def test_single_block_rejects_bad_arguments_without_a_gpu():
    """Validation happens on the host before any launch or device access."""
    from fireprot_b200 import _lib, modules
    lib = _lib.load()
    assert lib.fpb_single_block_workspace_size(64, 64, 256) == 0
    assert lib.fpb_single_block_workspace_size(64, 65, 384) == 0
    assert lib.fpb_single_block_workspace_size(0, 0, 384) == 0
    need = lib.fpb_single_block_workspace_size(1536, 1536, 384)
    assert need > 16 * 1536 * 1536 * 4  # the transposed pair bias
    w = modules.SingleBlockWeights(*([4096] * 16))
    ws = 1 << 20
    assert lib.fpb_single_block(None, None, None, 8, 8, 0, 384, ctypes.byref(w), 1e-5, 0, None,
                                0, None) == 4
    args = (4096, 4096, None)
    assert lib.fpb_single_block(*args, 8, 8, 0, 256, ctypes.byref(w), 1e-5, 0, ws, 1 << 30,
                                None) == 2                      # c_s
    assert lib.fpb_single_block(*args, 8, 4, 6, 384, ctypes.byref(w), 1e-5, 0, ws, 1 << 30,
                                None) == 2                      # r0 + rows > n
    assert lib.fpb_single_block(*args, 8, 8, 0, 384, ctypes.byref(w), 1e-5, 3, ws, 1 << 30,
                                None) == 4                      # precision
    assert lib.fpb_single_block(4104, 4096, None, 8, 8, 0, 384, ctypes.byref(w), 1e-5, 0, ws,
                                1 << 30, None) == 3             # misaligned s
    assert lib.fpb_single_block(*args, 8, 8, 0, 384, ctypes.byref(w), 1e-5, 0, ws, 1024,
                                None) == 7                      # workspace
    w.w_k = None
    assert lib.fpb_single_block(*args, 8, 8, 0, 384, ctypes.byref(w), 1e-5, 0, ws, 1 << 30,
                                None) == 4
