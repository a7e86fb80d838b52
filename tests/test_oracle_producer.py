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
