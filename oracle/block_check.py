"""Line-sampled parity of a whole Pairformer block at full size.

TEST INFRASTRUCTURE ONLY (``tests/`` and the CPU leg of ``bench.py``): the
checker, never the thing measured. Given the pair tensor before and after
each operator of a block as computed on the GPU, it recomputes a few lines
of each operator's output with the row-sampled oracle forms
(``pairformer_oracle.trimul_rows`` / ``triattn_lines`` / ``transition_rows``
/ ``single_block_rows``) from the GPU's own input to that operator, so every
operator of the chain is checked at the timed size without running the
full-size CPU restatement.

Lines are rows, except for the ending-node attention, whose update is
checked on columns (row l of the starting-node form on z^T).
"""
from __future__ import annotations

import torch

from . import pairformer_oracle as O

PAIR_OPERATORS = ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end",
                  "pair_transition")


def _cpu(t):
    return None if t is None else t.detach().to("cpu", torch.float32)


def params_from_weights(pair_weights: dict, single_weights: dict | None = None):
    """Oracle parameters from the weight dicts of ``PairformerPairBlock``'s
    operators (``{name: module.weight_dict()}``) and the single stack's
    ``weight_dict()`` (CPU float32 copies)."""
    def tm(w):
        return O.TriMulParams(**{k: _cpu(v) for k, v in w.items()})

    def ta(w):
        return O.TriAttnParams(heads=4, head_dim=32, **{k: _cpu(v) for k, v in w.items()})

    pw = pair_weights
    pair = O.PairBlockParams(
        tm(pw["tri_mul_out"]), tm(pw["tri_mul_in"]), ta(pw["tri_att_start"]),
        ta(pw["tri_att_end"]),
        O.TransitionParams(**{k: _cpu(v) for k, v in pw["pair_transition"].items()}))
    single = None
    if single_weights is not None:
        w = single_weights
        tr = O.TransitionParams(ln_w=_cpu(w["tr_ln_w"]), ln_b=_cpu(w["tr_ln_b"]),
                                w_a=_cpu(w["tr_w_a"]), w_b=_cpu(w["tr_w_b"]),
                                w_out=_cpu(w["tr_w_out"]))
        single = O.SingleBlockParams(heads=16, head_dim=24, transition=tr, **{
            k: _cpu(w[k]) for k in ("ln_a_w", "ln_a_b", "w_q", "b_q", "w_k", "w_v", "w_g",
                                    "w_o", "ln_z_w", "ln_z_b", "w_z")})
    return pair, single


def compared_lines(name: str, z, lines):
    """The lines of ``z`` that operator ``name`` is checked on."""
    idx = torch.as_tensor(lines, dtype=torch.long)
    return z[:, idx].transpose(0, 1) if name == "tri_att_end" else z[idx]


def expected_lines(name: str, z_in, mask, p: "O.PairBlockParams", lines):
    """Those lines of ``z_in + operator(z_in)`` from the oracle."""
    if name == "tri_mul_out":
        return O.trimul_rows(z_in, mask, p.tri_mul_out, lines, outgoing=True)
    if name == "tri_mul_in":
        return O.trimul_rows(z_in, mask, p.tri_mul_in, lines, outgoing=False)
    if name in ("tri_att_start", "tri_att_end"):
        start = name == "tri_att_start"
        pa = p.tri_att_start if start else p.tri_att_end
        return (compared_lines(name, z_in, lines)
                + O.triattn_lines(z_in, mask, pa, lines, starting=start))
    if name == "pair_transition":
        return O.transition_rows(z_in, p.transition, lines)
    raise ValueError(name)


def line_errors(got, ref, base) -> dict:
    """Output-scale relative errors of the result and of the update alone."""
    return {"out": O.rel_max_err(got, ref), "update": O.rel_max_err(got - base, ref - base)}


def check_pair_operator(name: str, z_in, z_out, mask, p, lines) -> dict:
    """Errors of one pair operator's GPU result ``z_out`` (host copy) on
    ``lines``, given the GPU's input ``z_in`` (host copy)."""
    ref = expected_lines(name, z_in, mask, p, lines)
    return line_errors(compared_lines(name, z_out, lines), ref, compared_lines(name, z_in, lines))


def check_single(s_in, s_out, z, mask, ps, lines) -> dict:
    """Errors of the single stack's GPU result on ``lines`` (rows of s)."""
    idx = torch.as_tensor(lines, dtype=torch.long)
    ref = O.single_block_rows(s_in, z, mask, ps, lines)
    return line_errors(s_out[idx], ref, s_in[idx])
