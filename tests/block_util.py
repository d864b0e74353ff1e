"""Test helper: copy a ``fireprot_b200.modules.PairformerPairBlock`` into the
oracle's parameter dataclasses (CPU float32)."""
from oracle import pairformer_oracle as O


def _c(t):
    return None if t is None else t.detach().float().cpu()


def trimul_params(m):
    w = m.weight_dict()
    return O.TriMulParams(**{k: _c(v) for k, v in w.items()})


def triattn_params(m):
    w = m.weight_dict()
    return O.TriAttnParams(heads=m.no_heads, head_dim=m.c_hidden, **{k: _c(v) for k, v in w.items()})


def transition_params(m):
    return O.TransitionParams(**{k: _c(v) for k, v in m.weight_dict().items()})


def block_params(b):
    return O.PairBlockParams(trimul_params(b.tri_mul_out), trimul_params(b.tri_mul_in),
                             triattn_params(b.tri_att_start), triattn_params(b.tri_att_end),
                             transition_params(b.pair_transition))
