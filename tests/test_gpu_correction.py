"""GPU parity of the bias rectification (inference): bsa_rectified_sparse_attn /
bsa_taylor_sparse_attn (bias_rectification.py:261-446) through the CUDA library.

* raw chunk scores, R_n, M, the unselected-chunk words and A_pool on them are
  bit-exact against the CPU oracle (same operation order), which
  tests/test_oracle_correction.py pins to the reference;
* the corrected output matches the float64 restatement and the reference's
  stored rows within max-abs 2e-2 and relative L2 1e-2;
* the unpadded dispatch (run_bsa_uniform(correction=...)) equals the
  reference-signature entry on the padded chunk-ordered tensors;
* the path refuses to run when gradients are required.
"""
import numpy as np
import pytest
import torch

from helpers import rel_l2
from inputs import CORRECTION_CASES, make_inputs
from oracle import oracle as O
from prism_b200 import _lib, bsa_rectified_sparse_attn, bsa_taylor_sparse_attn, ops, run_bsa_uniform
from prism_b200.bsa_interface import build_uniform_plan
from test_oracle_correction import chunk_valid, col_scale, corrected_output, stats
from test_oracle_uniform import _setup

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref).max()
    r = rel_l2(got, ref)
    assert err <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {r:.3e}"


def _entry(case):
    c = case.correction
    return bsa_taylor_sparse_attn if c["kind"] == "taylor" else bsa_rectified_sparse_attn


def _chunk_ordered(case, r, cuda):
    """The reference's inputs: q / k / v in the 3D-chunk order, key mask likewise."""
    inp = make_inputs(case)
    src_q = torch.as_tensor(r["src_q"], device=cuda).long()
    src_k = torch.as_tensor(r["src_k"], device=cuda).long()
    q = inp["q"].to(cuda)[:, :, src_q]
    k = inp["k"].to(cuda)[:, :, src_k]
    v = inp["v"].to(cuda)[:, :, src_k]
    vm = None if inp["valid"] is None else inp["valid"].to(cuda)[src_k]
    return q, k, v, vm


def _kw(case, r, cuda):
    c = case.correction
    kw = dict(chunk_size_q=r["cq"], chunk_size_k=r["ck"], sparsity=case.sparsity,
              cdf_threshold=case.cdf_threshold, sm_scale=1.0 / case.head_dim ** 0.5)
    cs = col_scale(r)
    if cs is not None:
        kw["score_modifier"] = torch.as_tensor(cs, device=cuda).view(1, 1, 1, -1)
    if c["kind"] == "taylor":
        kw["alpha_f"] = c["alpha_f"]
    return kw


@pytest.mark.parametrize("name", list(CORRECTION_CASES))
def test_correction_stats_bit_exact(name, cuda):
    case = CORRECTION_CASES[name]
    inp = make_inputs(case)
    r = _setup(name)
    gp = case.grid_padded
    valid = None if inp["valid"] is None else inp["valid"].to(cuda)
    plan = build_uniform_plan(gp, gp, case.chunk_q, case.chunk_k, case.head_dim, cuda,
                              sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                              valid_mask=valid)
    q_re = ops.gather_rows(inp["q"][0].to(cuda), gp, gp, plan.src_idx)
    k_re = ops.gather_rows(inp["k"][0].to(cuda), gp, gp, plan.src_idx_k)
    cs = col_scale(r)
    u = plan.uniform
    bq, _, pooled = ops.block_select_uniform(
        q_re, k_re, u["seq_q"], u["seq_k"], u["chunk_q"], u["chunk_k"], u["q_bits"], plan.tile_bits,
        case.sparsity, case.cdf_threshold,
        col_scale=None if cs is None else torch.as_tensor(cs, device=cuda), want_pooled=True)
    scores = ops.chunk_scores(pooled["qc"], pooled["kc"])
    S, nk = r["S"], r["S"] // r["ck"]
    # the selection at chunk level (first tile of each chunk pair)
    dense = O.bits_to_dense(bq.cpu().numpy().view(np.uint32), q_re.shape[1] // 64)
    tq, tk = r["cq"] // 64, r["ck"] // 64
    sel = dense[:, ::tq][:, :S // r["cq"], :nk * tk].reshape(case.heads, -1, nk, tk).any(-1)
    sel &= chunk_valid(r)[None, None, :]
    st = stats(r, sel)
    assert np.array_equal(scores.cpu().numpy().view(np.uint32), st["scores"].view(np.uint32))
    R, M, nonsel, a_rect = ops.correction_stats(scores, bq, plan.tile_bits, tq, tk,
                                                1.0 / case.head_dim ** 0.5, want_nonsel=True,
                                                want_a_rect=True)
    for got, ref in ((R, st["R"]), (M, st["M"]), (a_rect, st["a_rect"])):
        assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(nonsel.cpu().numpy().view(np.uint64), st["nonsel"])


@pytest.mark.parametrize("name", list(CORRECTION_CASES))
def test_correction_output_parity(name, cuda):
    case = CORRECTION_CASES[name]
    r = _setup(name)
    fx = r["fx"]
    q, k, v, vm = _chunk_ordered(case, r, cuda)
    with torch.no_grad():
        out = _entry(case)(q, k, v, kv_valid_mask=vm, **_kw(case, r, cuda))
    assert _lib.load().prism_device_status() == 0
    got = out[0].float().cpu().numpy()
    # float64 restatement on the oracle's selection (== the CUDA selection)
    nk = r["S"] // r["ck"]
    _, _, sel = O.block_select_uniform(r["q"][:, r["src_q"]], r["k"][:, r["src_k"]], r["S"], r["S"],
                                       r["cq"], r["ck"], r["valid_re"], r["valid_re"],
                                       case.sparsity, case.cdf_threshold, want_chunks=True,
                                       col_scale=col_scale(r))
    sel = sel.astype(bool)
    ref = corrected_output(r, sel, stats(r, sel))
    _close(got, ref, "output vs oracle")
    _close(got[:, fx["rows"]], fx["o"], "output vs reference")


@pytest.mark.parametrize("name", ["r_rect_pad", "r_taylor_pad"])
def test_run_bsa_uniform_correction(name, cuda):
    """The unpadded dispatch equals the reference-signature entry on the padded,
    chunk-ordered tensors (scattered back to THW), bit for bit."""
    case = CORRECTION_CASES[name]
    r = _setup(name)
    inp = make_inputs(case)
    q, k, v, vm = _chunk_ordered(case, r, cuda)
    c = case.correction
    with torch.no_grad():
        ref = _entry(case)(q, k, v, kv_valid_mask=vm, **_kw(case, r, cuda))
        qu, ku, vu = (inp[n + "_u"].to(cuda) for n in ("q", "k", "v"))
        out = run_bsa_uniform(qu, ku, vu, case.grid, sparsity=case.sparsity,
                              cdf_threshold=case.cdf_threshold, chunk_3d_shape_q=case.chunk_q,
                              chunk_3d_shape_k=case.chunk_k, correction=c["kind"],
                              taylor_alpha_f=c.get("alpha_f", 0.5))
    inv = torch.as_tensor(r["inv_q"], device=cuda).long()
    ref_thw = ref[:, :, inv]
    T, H, W = case.grid
    h, D = case.heads, case.head_dim
    ref_u = ref_thw.view(1, h, *case.grid_padded, D)[:, :, :T, :H, :W].reshape(1, h, T * H * W, D)
    assert torch.equal(out, ref_u)


def test_correction_refuses_grad(cuda):
    q = torch.zeros(1, 2, 512, 64, dtype=torch.bfloat16, device=cuda, requires_grad=True)
    with pytest.raises(NotImplementedError):
        bsa_taylor_sparse_attn(q, q, q, 64, 64, 0.5, None, 0.125)


def test_rectified_contraction_fixed_order(cuda):
    """prism_rectified_contract (the Rectified form's A_rect V_cmp) against a float64
    product, on sizes that leave partial tiles in every dimension, and run-to-run
    bit-identical."""
    g = torch.Generator().manual_seed(21)
    heads, nq, nk, D = 3, 97, 150, 128
    a = (torch.rand(heads, nq, nk, generator=g) * (torch.rand(heads, nq, nk, generator=g) < 0.4)).to(cuda)
    v = torch.randn(heads, nk, D, generator=g).to(cuda)
    got = ops.rectified_contract(a, v)
    ref = torch.bmm(a.double(), v.double())
    assert float((got.double() - ref).abs().max()) <= 1e-5 * max(1.0, float(ref.abs().max()))
    assert torch.equal(got, ops.rectified_contract(a, v))
