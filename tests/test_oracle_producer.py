"""Pin the producer-side restatement (RMSNorm + 3D RoPE, wan_video_dit.py:699-705)
against golden vectors made by the reference's own precompute_freqs_cis_3d and
rope_apply_head_dim (taken from its source by tests/golden/make_golden.py) and
torch.nn.RMSNorm (the module SelfAttention uses).

* prism_b200.producer.rope_table equals the reference's frequency table bit for bit;
* the RoPE restatement reproduces rope_apply_head_dim bit for bit on the reference's
  normed values;
* the RMSNorm restatement is within one bf16 unit of torch.nn.RMSNorm (torch leaves
  the reduction order of the mean unspecified) and equal on nearly every element.
"""
import numpy as np
import pytest

from helpers import load_fixture
from inputs import PRODUCER_CASES, make_producer_inputs
from oracle import oracle as O
from prism_b200.producer import rope_table


def _b(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("name", list(PRODUCER_CASES))
def test_rope_table_matches_reference(name):
    grid, heads, D, seed = PRODUCER_CASES[name]
    fx = load_fixture(name)
    t = rope_table(grid, D).numpy()
    assert t.shape == fx["freqs"].shape
    assert np.array_equal(t.view(np.uint64), fx["freqs"].view(np.uint64))


@pytest.mark.parametrize("name", list(PRODUCER_CASES))
def test_rope_restatement_bit_exact(name):
    grid, heads, D, seed = PRODUCER_CASES[name]
    fx = load_fixture(name)
    y = O.rope_apply(fx["normed"], fx["freqs"], D)
    assert np.array_equal(y, fx["y"])


@pytest.mark.parametrize("name", list(PRODUCER_CASES))
def test_rms_norm_restatement(name):
    grid, heads, D, seed = PRODUCER_CASES[name]
    fx = load_fixture(name)
    x, gamma = make_producer_inputs(grid, heads, D, seed)
    got = O.rms_norm(_b(x[0]), gamma.float().numpy())
    ref = fx["normed"]
    diff = np.abs(got.astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() >= 0.99, (diff.max(), (diff == 0).mean())


def _ff_dot2(a, chi, clo, b, shi, slo, sign):
    """The kernels' float-float a c + sign b s, emulated exactly: each fmaf's exact
    value is representable in float64 (a bf16 times a float needs <= 32 bits), so
    float64 arithmetic rounded once to float32 is the fused multiply-add."""
    f32 = np.float32
    a, b = a.astype(f32), (sign * b).astype(f32)
    p1 = (a * chi).astype(f32)
    e1 = (a.astype(np.float64) * clo + ((a.astype(np.float64) * chi) - p1).astype(f32)).astype(f32)
    p2 = (b * shi).astype(f32)
    e2 = (b.astype(np.float64) * slo + ((b.astype(np.float64) * shi) - p2).astype(f32)).astype(f32)
    s = (p1 + p2).astype(f32)
    bb = (s - p1).astype(f32)
    err = ((p1 - (s - bb).astype(f32)).astype(f32) + (p2 - bb).astype(f32)).astype(f32)
    return (s + (err + (e1 + e2).astype(f32)).astype(f32)).astype(f32)


def test_float_float_rotation_matches_double():
    """The kernels' float-float rotation rounds to the same bf16 as the reference's
    double evaluation (rounded through float) on random bf16 pairs and angles."""
    rng = np.random.default_rng(0)
    n = 1 << 20
    a = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32) * 3))
    b = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32) * 3))
    ang = rng.uniform(0, 1000.0, n)
    c, s = np.cos(ang), np.sin(ang)
    chi, shi = c.astype(np.float32), s.astype(np.float32)
    clo = (c - chi.astype(np.float64)).astype(np.float32)
    slo = (s - shi.astype(np.float64)).astype(np.float32)
    for got, ref in ((_ff_dot2(a, chi, clo, b, shi, slo, -1.0), a * c - b * s),
                     (_ff_dot2(a, shi, slo, b, chi, clo, 1.0), a * s + b * c)):
        g16 = O.f32_to_bf16_bits(got)
        r16 = O.f32_to_bf16_bits(ref.astype(np.float32))
        assert np.array_equal(g16, r16), int((g16 != r16).sum())
