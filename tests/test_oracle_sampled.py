"""The row-sampled oracle forms against the full oracle (CPU).

The full-size GPU parity tests and the bench's parity check compare CUDA
results with ``trimul_rows`` / ``triattn_lines`` / ``transition_rows`` /
``single_block_rows`` on a few lines; here those forms are held to the full
operators (which ``test_oracle_golden.py`` pins to the reference) in float64
on small, ragged, masked cases, and the all -inf row semantics of
``attention_core`` are pinned to torch's softmax and
``scaled_dot_product_attention``.
"""
import pytest
import torch

from oracle import pairformer_oracle as O

F64 = torch.float64


def _mask(n, kind):
    if kind == "none":
        return None
    if kind == "padding":
        return O.make_padding_mask(n, n - 3, dtype=F64)
    g = torch.Generator().manual_seed(4)
    m = (torch.rand(n, n, generator=g) > 0.3).to(F64)
    m[1, :] = 0.0
    m[:, 2] = 0.0
    return m


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("mask_kind", ["none", "random", "padding"])
def test_trimul_rows_match_full(outgoing, mask_kind):
    n = 23
    z = O.make_pair(n, seed=5, dtype=F64)
    p = O.make_trimul_params(seed=6, dtype=F64, ln_affine_random=True)
    mask = _mask(n, mask_kind)
    rows = O.sample_lines(n, count=5, seed=1, valid=n - 3)
    for add in (True, False):
        full = O.triangle_multiplication(z, mask, p, outgoing=outgoing, add=add)
        part = O.trimul_rows(z, mask, p, rows, outgoing=outgoing, add=add)
        assert torch.allclose(part, full[rows], rtol=0, atol=1e-12)


@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("mask_kind", ["none", "random", "padding"])
def test_triattn_lines_match_full(starting, mask_kind):
    n = 21
    z = O.make_pair(n, seed=7, dtype=F64)
    p = O.make_triattn_params(seed=8, dtype=F64, with_biases=True, ln_affine_random=True)
    mask = _mask(n, mask_kind)
    lines = O.sample_lines(n, count=6, seed=2, valid=n - 3)
    full = O.triangle_attention(z, mask, p, starting=starting, chunk=5)
    part = O.triattn_lines(z, mask, p, lines, starting=starting, chunk=3)
    expect = full[lines] if starting else full[:, lines].transpose(0, 1)
    assert torch.allclose(part, expect, rtol=0, atol=1e-12)


def test_transition_and_single_rows_match_full():
    n = 19
    z = O.make_pair(n, seed=9, dtype=F64)
    s = O.make_single(n, seed=10, dtype=F64)
    mask = O.make_padding_mask(n, n - 4, dtype=F64)
    pt = O.make_transition_params(seed=11, dtype=F64, ln_affine_random=True)
    ps = O.make_single_params(seed=12, dtype=F64, ln_affine_random=True)
    rows = O.sample_lines(n, count=4, seed=3, valid=n - 4)
    full_t = z + O.pair_transition(z, pt)
    assert torch.allclose(O.transition_rows(z, pt, rows), full_t[rows], rtol=0, atol=1e-12)
    full_s = O.single_block(s, z, mask, ps)
    assert torch.allclose(O.single_block_rows(s, z, mask, ps, rows), full_s[rows], rtol=0,
                          atol=1e-12)


def test_sample_lines_include_the_edges():
    rows = O.sample_lines(1536, count=12, seed=0, valid=1480)
    assert rows == sorted(set(rows))
    assert {0, 1479, 1480, 1535} <= set(rows)
    assert len(rows) >= 14


def test_attention_core_empty_rows():
    """A query row with every logit -inf: NaN through softmax (upstream
    ``_attention``), 0 through ``scaled_dot_product_attention`` (the
    Protenix dispatch's reference); other rows identical in both."""
    g = torch.Generator().manual_seed(521)
    q, k, v = (torch.randn(3, 4, 9, 32, generator=g) for _ in range(3))
    bias = torch.randn(1, 4, 9, 9, generator=g)
    bias[:, :, 0, :] = float("-inf")
    bias[:, :, 1, 0] = 80.0
    soft = O.attention_core(q, k, v, [bias])
    zero = O.attention_core(q, k, v, [bias], empty_rows="zero")
    assert torch.isnan(soft[:, :, 0]).all()
    assert (zero[:, :, 0] == 0).all()
    assert torch.equal(soft[:, :, 1:], zero[:, :, 1:])
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=bias, scale=1.0)
    assert torch.allclose(zero, sdpa, rtol=2e-5, atol=2e-5)
