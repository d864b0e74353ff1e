"""CPU timing of the reference's native pair-path math (oracle port).

TEST / BASELINE INFRASTRUCTURE ONLY (used by ``bench.py``'s CPU-baseline leg
and its ``--impl reference`` arm). Two forms:

``FullBlock``: one whole Pairformer block, every stage in full (no sampling,
no scaling), as an ordered list of work items that a caller can split over
several timed steps; the reference arm times exactly one such block.

``sampled_block_seconds``: a bounded sample of one Pairformer block, timed
with the same torch operations as ``pairformer_oracle`` on the host cores:

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


# ---------------------------------------------------------------------------
# one whole block, unsampled, as ordered work items
# ---------------------------------------------------------------------------
class FullBlock:
    """One whole Pairformer block of the native math at size n (pair stack,
    then the single stack), every stage computed in full, as an ordered list
    of work items ``(label, flops, fn)`` that must run in order. The O(N^3)
    stages are split into slices (``chan_chunk`` contraction channel planes,
    ``row_chunk`` attention rows, as the reference's own outer-chunk loop,
    ``triangle_attention.py:113-128``) so that consecutive items can be
    grouped into timed steps of similar length; the slices together compute
    exactly the unsliced stage."""

    def __init__(self, n: int, valid: int | None = None, *, seed: int = 0,
                 row_chunk: int = 32, chan_chunk: int = 8):
        self.n = n
        self.z = O.make_pair(n, seed=seed)
        self.mask = O.make_padding_mask(n, valid if valid is not None else n)
        self.p = O.make_block_params(seed=seed + 1)
        self.s = O.make_single(n, seed=seed + 2)
        self.ps = O.make_single_params(seed=seed + 3)
        self.st = {}
        self.items = []
        c = 128
        n2 = float(n) * n
        for name, p, outgoing in (("tri_mul_out", self.p.tri_mul_out, True),
                                  ("tri_mul_in", self.p.tri_mul_in, False)):
            self.items.append((f"{name}.proj", 2 * n2 * c * 5 * c,
                               lambda p=p: self._tm_proj(p)))
            for c0 in range(0, c, chan_chunk):
                self.items.append((f"{name}.contract[{c0}]", 2 * n2 * n * chan_chunk,
                                   lambda c0=c0, o=outgoing: self._tm_contract(c0, chan_chunk, o)))
            self.items.append((f"{name}.out", 2 * n2 * c * c, lambda p=p: self._tm_out(p)))
        for name, p, starting in (("tri_att_start", self.p.tri_att_start, True),
                                  ("tri_att_end", self.p.tri_att_end, False)):
            self.items.append((f"{name}.proj", 2 * n2 * c * (4 * c + 4),
                               lambda p=p, st=starting: self._ta_proj(p, st)))
            for r0 in range(0, n, row_chunk):
                rows = min(row_chunk, n - r0)
                self.items.append((f"{name}.core[{r0}]", 4 * rows * n2 * c,
                                   lambda r0=r0, rows=rows: self._ta_core(r0, rows)))
            self.items.append((f"{name}.out", 2 * n2 * c * c,
                               lambda p=p, st=starting: self._ta_out(p, st)))
        for r0 in range(0, n, row_chunk * 8):
            rows = min(row_chunk * 8, n - r0)
            self.items.append((f"pair_transition[{r0}]", 2.0 * rows * n * 12 * c * c,
                               lambda r0=r0, rows=rows: self._transition(r0, rows)))
        self.items.append(("single", 5632.0 * n2, self._single))

    # -- triangle multiplication
    def _tm_proj(self, p):
        zn = O.layer_norm(self.z, p.ln_in_w, p.ln_in_b)
        m = self.mask[..., None]
        a = torch.sigmoid(zn @ p.w_a_g.T) * (zn @ p.w_a_p.T) * m
        b = torch.sigmoid(zn @ p.w_b_g.T) * (zn @ p.w_b_p.T) * m
        self.st = {"a": a.permute(2, 0, 1).contiguous(), "b": b.permute(2, 0, 1).contiguous(),
                   "g": torch.sigmoid(zn @ p.w_g.T),
                   "x": torch.empty(128, self.n, self.n)}

    def _tm_contract(self, c0, cc, outgoing):
        a, b = self.st["a"][c0:c0 + cc], self.st["b"][c0:c0 + cc]
        if outgoing:
            self.st["x"][c0:c0 + cc] = torch.matmul(a, b.transpose(-1, -2))
        else:
            self.st["x"][c0:c0 + cc] = torch.matmul(a.transpose(-1, -2), b)

    def _tm_out(self, p):
        x = O.layer_norm(self.st["x"].permute(1, 2, 0), p.ln_out_w, p.ln_out_b) @ p.w_z.T
        self.z = self.z + self.st["g"] * x
        self.st = {}

    # -- triangle attention
    def _ta_proj(self, p, starting):
        n, H, d = self.n, p.heads, p.head_dim
        x = self.z if starting else self.z.transpose(0, 1)
        m = self.mask if starting else self.mask.transpose(0, 1)
        xn = O.layer_norm(x, p.ln_w, p.ln_b)
        gate = xn @ p.w_g.T
        if p.b_g is not None:
            gate = gate + p.b_g
        self.st = {
            "q": (xn @ p.w_q.T).reshape(n, n, H, d).permute(0, 2, 1, 3) * (d ** -0.5),
            "k": (xn @ p.w_k.T).reshape(n, n, H, d).permute(0, 2, 1, 3),
            "v": (xn @ p.w_v.T).reshape(n, n, H, d).permute(0, 2, 1, 3),
            "tb": (xn @ p.w_bias.T).permute(2, 0, 1).unsqueeze(0),
            "gate": torch.sigmoid(gate), "m": m, "o": torch.empty(n, n, H * d)}

    def _ta_core(self, r0, rows):
        st = self.st
        sl = slice(r0, r0 + rows)
        mb = (O.MASK_INF * (st["m"][sl] - 1.0))[:, None, None, :]
        o = O.attention_core(st["q"][sl], st["k"][sl], st["v"][sl], [mb, st["tb"]])
        st["o"][sl] = o.permute(0, 2, 1, 3).reshape(rows, self.n, -1)

    def _ta_out(self, p, starting):
        out = (self.st["gate"] * self.st["o"]) @ p.w_o.T
        if p.b_o is not None:
            out = out + p.b_o
        self.z = self.z + (out if starting else out.transpose(0, 1))
        self.st = {}

    # -- transition, single stack
    def _transition(self, r0, rows):
        if r0 == 0:
            self.st = {"z": self.z.clone()}
        sl = slice(r0, r0 + rows)
        self.st["z"][sl] += O.pair_transition(self.z[sl], self.p.transition)
        if r0 + rows >= self.n:
            self.z = self.st["z"]
            self.st = {}

    def _single(self):
        self.s = O.single_block(self.s, self.z, self.mask, self.ps)

    def steps(self, k: int):
        """Consecutive groups of items, k groups of roughly equal FLOPs."""
        total = sum(f for _, f, _ in self.items)
        groups = [[] for _ in range(k)]
        acc = 0.0
        for item in self.items:
            g = min(k - 1, int(acc / total * k))
            groups[g].append(item)
            acc += item[1]
        return groups
