"""Pin the CPU oracle's bias rectification (inference) against golden vectors
produced by the reference's own ``bsa_rectified_sparse_attn`` and
``bsa_taylor_sparse_attn`` (bias_rectification.py:261-446, PyTorch merge, run on
CPU under no_grad by tests/golden/make_golden.py).

* the chunk selection (with the score modifier of the modifier case) equals the
  reference's;
* R_n and the variance M of A_pool agree with the reference's fp32 values to
  float32 rounding, and the flat / sharp split (M < quantile(M, alpha_f)) is
  the reference's;
* the corrected output, restated in float64 on the reference's selection,
  matches the reference's on the stored rows.
"""
import numpy as np
import pytest

from inputs import CORRECTION_CASES
from oracle import oracle as O
from test_oracle_uniform import _bits_from_chunks, _setup, _tie_free_chunks


def chunk_valid(r):
    nk = r["S"] // r["ck"]
    if r["valid_re"] is None:
        return np.ones(nk, bool)
    return r["valid_re"].reshape(nk, r["ck"]).any(axis=1)


def col_scale(r):
    c = r["case"].correction
    if c.get("variance_gamma", 0.0) <= 0:
        return None
    rho = O.variance_density(r["v"][:, r["src_k"]], r["S"], r["case"].chunk_k, r["valid_re"])
    return O.guidance_scale(r["S"] // r["ck"], rho, c["variance_gamma"])


def stats(r, sel):
    """Oracle raw scores, pooled chunks and correction statistics on a selection."""
    qc, kc, sc = O.uniform_pooled(r["q"][:, r["src_q"]], r["k"][:, r["src_k"]], r["S"], r["S"],
                                  r["cq"], r["ck"], r["valid_re"], r["valid_re"])
    sm = 1.0 / np.sqrt(r["case"].head_dim)
    R, M, nonsel, a_rect = O.correction_stats(sc, sel, chunk_valid(r), sm, want_a_rect=True)
    return dict(qc=qc, kc=kc, scores=sc, R=R, M=M, nonsel=nonsel, a_rect=a_rect, sm=sm)


def v_pooled(r):
    v = O.bf16_bits_to_f32(r["v"][:, r["src_k"]]).astype(np.float64)
    nk = r["S"] // r["ck"]
    w = np.ones(r["S"]) if r["valid_re"] is None else r["valid_re"].astype(np.float64)
    num = (v * w[None, :, None]).reshape(v.shape[0], nk, r["ck"], -1).sum(2)
    den = np.maximum(w.reshape(nk, r["ck"]).sum(1), 1.0)
    return num / den[None, :, None]


def corrected_output(r, sel_dense, st):
    """float64 restatement of the corrected output (rows in chunk order)."""
    case = r["case"]
    f = O.bf16_bits_to_f32
    qr, kr, vr = f(r["q"][:, r["src_q"]]), f(r["k"][:, r["src_k"]]), f(r["v"][:, r["src_k"]])
    bq = _bits_from_chunks(sel_dense, r)
    o, lse = O.bsa_forward(qr, kr, vr, bq, r["valid_re"])
    vc = v_pooled(r)
    if case.correction["kind"] == "rectified":
        return O.rectified_output(o, st["R"], st["a_rect"], vc, r["cq"])
    tau = np.float32(np.quantile(st["M"].astype(np.float64).reshape(-1), case.correction["alpha_f"]))
    flat = st["M"] < tau
    nk = r["S"] // r["ck"]
    cnt = (np.full(nk, r["ck"]) if r["valid_re"] is None
           else r["valid_re"].reshape(nk, r["ck"]).sum(1))
    nonsel = ~sel_dense & chunk_valid(r)[None, None, :]
    return O.taylor_output(qr, o, lse, st["kc"], vc, nonsel, flat,
                           np.log(np.maximum(cnt, 1)).astype(np.float64), r["cq"], st["sm"])


@pytest.mark.parametrize("name", list(CORRECTION_CASES))
def test_correction_selection_matches_reference(name):
    r = _setup(name)
    nk = r["S"] // r["ck"]
    _, _, sel = O.block_select_uniform(r["q"][:, r["src_q"]], r["k"][:, r["src_k"]], r["S"], r["S"],
                                       r["cq"], r["ck"], r["valid_re"], r["valid_re"],
                                       r["case"].sparsity, r["case"].cdf_threshold, want_chunks=True,
                                       col_scale=col_scale(r))
    ref = O.bits_to_dense(r["fx"]["sel_chunks_f32"], nk)
    ok = _tie_free_chunks(r)
    assert (sel.astype(bool)[:, ok] == ref[:, ok]).all()


@pytest.mark.parametrize("name", list(CORRECTION_CASES))
def test_correction_stats_match_reference(name):
    r = _setup(name)
    fx = r["fx"]
    sel = O.bits_to_dense(fx["sel_chunks_f32"], r["S"] // r["ck"])
    st = stats(r, sel)
    np.testing.assert_allclose(st["R"], fx["R"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(st["M"], fx["M"], rtol=1e-4, atol=1e-9)
    if r["case"].correction["kind"] == "taylor":
        tau = float(fx["tau"])
        mine = st["M"] < np.float32(np.quantile(st["M"].astype(np.float64).reshape(-1),
                                                r["case"].correction["alpha_f"]))
        ref = fx["M"] < tau
        # chunks far from the threshold take the reference's side
        far = np.abs(fx["M"] - tau) > 1e-5 * abs(tau)
        assert (mine[far] == ref[far]).all()
        assert ref.any() and (~ref).any()


@pytest.mark.parametrize("name", list(CORRECTION_CASES))
def test_correction_output_restatement(name):
    r = _setup(name)
    fx = r["fx"]
    sel = O.bits_to_dense(fx["sel_chunks_f32"], r["S"] // r["ck"])
    st = stats(r, sel)
    out = corrected_output(r, sel, st)
    got = out[:, fx["rows"]]
    ref = fx["o"]
    err = np.abs(got - ref).max()
    assert err <= 2e-5 * max(1.0, np.abs(ref).max()), err
