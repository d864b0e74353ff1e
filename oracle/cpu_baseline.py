"""Bounded CPU timing of the reference's native pair-path math (oracle port).

TEST / BASELINE INFRASTRUCTURE ONLY (used by ``bench.py``'s CPU-baseline leg
and its ``--impl reference`` arm). It times the same torch operations as
``pairformer_oracle`` on the host cores, on a bounded sample of one
Pairformer block:

- every O(N^2) stage (LayerNorms, all projections, gates, the transition)
  runs on the full N x N pair tensor;
- the O(N^3) stages run on a sample and are scaled linearly: the triangle
  contraction on ``chan_sample`` of the 128 channel planes, the triangle
  attention core (scores, mask/bias, softmax, P V) on ``row_sample`` rows i of
  N (the reference's own outer-chunk loop, ``triangle_attention.py:113-128``);
- the single stack (attention with pair bias over all N tokens, the single
  transition) runs in full.

Both directions of each operator have the same cost, so each is timed once
and counted twice. Returns seconds per block.
"""
from __future__ import annotations

import os
import time

import torch

from . import pairformer_oracle as O


def _timed(fn):
    t0 = time.perf_counter()
    out = fn()
    return out, time.perf_counter() - t0


def sampled_block_seconds(n: int = 1536, valid: int | None = None, *, row_sample: int = 16,
                          chan_sample: int = 8, threads: int | None = None, seed: int = 0,
                          single: bool = True):
    """Estimated seconds for one Pairformer block at size n (the single stack
    only when ``single``), and a breakdown."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    z = O.make_pair(n, seed=seed)
    mask = O.make_padding_mask(n, valid if valid is not None else n)
    p = O.make_block_params(seed=seed + 1)
    parts = {}
    with torch.no_grad():
        # --- triangle multiplication (one direction; x2)
        tm = p.tri_mul_out

        def tm_proj():
            zn = O.layer_norm(z, tm.ln_in_w, tm.ln_in_b)
            a = torch.sigmoid(zn @ tm.w_a_g.T) * (zn @ tm.w_a_p.T) * mask[..., None]
            b = torch.sigmoid(zn @ tm.w_b_g.T) * (zn @ tm.w_b_p.T) * mask[..., None]
            g = torch.sigmoid(zn @ tm.w_g.T)
            return a.permute(2, 0, 1).contiguous(), b.permute(2, 0, 1).contiguous(), g

        (a_cf, b_cf, g), t_proj = _timed(tm_proj)
        _, t_con = _timed(lambda: torch.matmul(a_cf[:chan_sample],
                                               b_cf[:chan_sample].transpose(-1, -2)))
        t_con *= 128.0 / chan_sample
        x = a_cf.permute(1, 2, 0)  # stands in for the contraction output (same shape)

        def tm_out():
            y = O.layer_norm(x, tm.ln_out_w, tm.ln_out_b) @ tm.w_z.T
            return z + g * y

        _, t_out = _timed(tm_out)
        del a_cf, b_cf, g, x
        parts["triangle_multiplication"] = 2 * (t_proj + t_con + t_out)

        # --- triangle attention (one direction; x2)
        ta = p.tri_att_start
        H, d = ta.heads, ta.head_dim

        def ta_proj():
            xn = O.layer_norm(z, ta.ln_w, ta.ln_b)
            q = (xn @ ta.w_q.T).reshape(n, n, H, d).permute(0, 2, 1, 3) * (d ** -0.5)
            k = (xn @ ta.w_k.T).reshape(n, n, H, d).permute(0, 2, 1, 3)
            v = (xn @ ta.w_v.T).reshape(n, n, H, d).permute(0, 2, 1, 3)
            tb = (xn @ ta.w_bias.T).permute(2, 0, 1).unsqueeze(0)
            gate = torch.sigmoid(xn @ ta.w_g.T)
            return q, k, v, tb, gate

        (q, k, v, tb, gate), t_aproj = _timed(ta_proj)
        r = min(row_sample, n)
        mb = (O.MASK_INF * (mask[:r] - 1.0))[:, None, None, :]
        o_s, t_core = _timed(lambda: O.attention_core(q[:r], k[:r], v[:r], [mb, tb]))
        t_core *= n / r
        o = torch.empty(n, n, H * d)
        o[:r] = o_s.permute(0, 2, 1, 3).reshape(r, n, H * d)

        def ta_out():
            return z + (gate * o) @ ta.w_o.T

        _, t_aout = _timed(ta_out)
        del q, k, v, tb, gate, o
        parts["triangle_attention"] = 2 * (t_aproj + t_core + t_aout)

        # --- transition
        _, t_tr = _timed(lambda: z + O.pair_transition(z, p.transition))
        parts["pair_transition"] = t_tr

        # --- single stack (AttentionPairBias + single transition), in full
        if single:
            s = O.make_single(n, seed=seed + 2)
            ps = O.make_single_params(seed=seed + 3)
            _, parts["single_stack"] = _timed(lambda: O.single_block(s, z, mask, ps))
    total = sum(parts.values())
    what = "one Pairformer block (pair and single stacks)" if single else "one pair block"
    sample = (f"{what} at N={n}: O(N^2) stages in full; triangle contraction on "
              f"{chan_sample}/128 channel planes and attention core on {r}/{n} rows, "
              f"scaled linearly; torch fp32 on {threads} host threads")
    return total, parts, sample, threads
