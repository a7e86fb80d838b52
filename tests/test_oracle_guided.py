"""Pin the CPU oracle's guided uniform path against golden vectors produced by
the reference's own ``flash_attn_bsa_3d_variance_guided`` (bsa_interface.py:
1179-1260) and ``flash_attn_bsa_3d_audio_guided`` (:1395-1501), run on CPU by
tests/golden/make_golden.py.

* the channel-variance density rho (compute_channel_variance_density,
  :973-1062), the audio block saliency (compute_block_audio_saliency,
  :1065-1102) and Path B's audio-weighted pooled keys
  (audio_weighted_mean_pooling_compression, :902-970) agree with the
  reference's fp32 values to float32 rounding (the reference leaves summation
  order to torch; the oracle fixes the order the CUDA kernels use);
* the chunk selection with the guidance scale (and Path B pooling) is identical
  to the reference's fp32 pass on every chunk whose pooled q is not all
  padding, and differs from the unguided selection (the cases exercise the
  guidance);
* on that selection the float64 attention restatement matches the reference's
  fp32 Triton outputs and gradients.

The reference's bf16 pass rounds rho and the scale to bf16 (rho.to(q.dtype),
:1243-1245, :1469) and, without a valid mask, pools and scores in bf16; its
selection may then differ from the fp32 pass near ties.  The agreement is
checked loosely.
"""
import numpy as np
import pytest

from inputs import GUIDED_CASES
from oracle import oracle as O
from test_oracle_uniform import _bits_from_chunks, _setup, _tie_free_chunks


def guidance(r):
    """Oracle rho, saliency, Path B weights and the per-key-chunk scale of a case."""
    case = r["case"]
    g = case.guidance
    S, ck = r["S"], r["ck"]
    vg = g.get("variance_gamma", 0.0)
    rho = O.variance_density(r["v"][:, r["src_k"]], S, case.chunk_k, r["valid_re"]) if vg > 0 else None
    sal = weights = None
    if g["kind"] == "audio":
        a = norms_re(r)
        sal = O.audio_saliency(a, S, ck, r["valid_re"])
        if g["lambda_w"] > 0:
            weights = O.audio_pool_weights(a, S, ck, r["valid_re"], g["lambda_w"])
    scale = O.guidance_scale(S // ck, rho, vg, sal, g.get("gate", 1.0), g.get("audio_gamma", 0.0))
    return dict(rho=rho, saliency=sal, weights=weights, scale=scale)


def norms_re(r):
    from inputs import make_inputs
    n = make_inputs(r["case"])["norms"].float().numpy()
    return n[r["src_k"]].astype(np.float32)


def select(r, gd, guided=True):
    case = r["case"]
    return O.block_select_uniform(r["q"][:, r["src_q"]], r["k"][:, r["src_k"]], r["S"], r["S"],
                                  r["cq"], r["ck"], r["valid_re"], r["valid_re"], case.sparsity,
                                  case.cdf_threshold, want_chunks=True,
                                  k_weights=gd["weights"] if guided else None,
                                  col_scale=gd["scale"] if guided else None)


@pytest.mark.parametrize("name", list(GUIDED_CASES))
def test_guidance_statistics_match_reference(name):
    r = _setup(name)
    gd = guidance(r)
    fx = r["fx"]
    if gd["rho"] is not None:
        np.testing.assert_allclose(gd["rho"], fx["rho"], rtol=2e-5, atol=1e-7)
        assert gd["rho"].max() == 1.0
    if gd["saliency"] is not None:
        np.testing.assert_allclose(gd["saliency"], fx["saliency"], rtol=2e-6, atol=1e-7)
    if gd["weights"] is not None:
        # Path B pooled keys from the oracle's weights, float64 sums
        k = O.bf16_bits_to_f32(r["k"][:, r["src_k"]]).astype(np.float64)
        w = gd["weights"].astype(np.float64)
        nk = r["S"] // r["ck"]
        kw = (k * w[None, :, None]).reshape(k.shape[0], nk, r["ck"], -1).sum(2)
        den = np.maximum(w.reshape(nk, r["ck"]).sum(1), 1.0)
        np.testing.assert_allclose(kw / den[None, :, None], fx["kcmp_pathb"], rtol=1e-5, atol=1e-6)
        if r["valid_re"] is not None:
            assert (gd["weights"][~r["valid_re"]] == 0).all()


@pytest.mark.parametrize("name", list(GUIDED_CASES))
def test_guided_selection_matches_reference(name):
    r = _setup(name)
    gd = guidance(r)
    nk = r["S"] // r["ck"]
    bits_q, bits_k, sel = select(r, gd)
    ref = O.bits_to_dense(r["fx"]["sel_chunks_f32"], nk)
    ok = _tie_free_chunks(r)
    mine = sel.astype(bool)
    assert (mine[:, ok] == ref[:, ok]).all(), f"{(mine[:, ok] != ref[:, ok]).sum()} chunk pairs differ"
    assert (bits_q == _bits_from_chunks(mine, r)).all()
    # the guidance matters on these inputs
    _, _, plain = select(r, gd, guided=False)
    assert (plain.astype(bool) != mine).any()
    # the reference's bf16 pass (bf16 scale, and bf16 scores without a mask)
    agree = (O.bits_to_dense(r["fx"]["sel_chunks"], nk) == ref)[:, ok].mean()
    assert agree >= 0.8, agree


@pytest.mark.parametrize("name", list(GUIDED_CASES))
def test_guided_attention_restatement(name):
    r = _setup(name)
    nk = r["S"] // r["ck"]
    bits_q = _bits_from_chunks(O.bits_to_dense(r["fx"]["sel_chunks_f32"], nk), r)
    f = O.bf16_bits_to_f32
    qr, kr, vr = f(r["q"][:, r["src_q"]]), f(r["k"][:, r["src_k"]]), f(r["v"][:, r["src_k"]])
    o, _ = O.bsa_forward(qr, kr, vr, bits_q, r["valid_re"])
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, f(r["do"])[:, r["src_q"]], bits_q, r["valid_re"])
    fx, rows = r["fx"], r["fx"]["rows"]
    for nm, x, inv in (("o", o, r["inv_q"]), ("dq", dq, r["inv_q"]), ("dk", dk, r["inv_k"]),
                       ("dv", dv, r["inv_k"])):
        got = x[:, inv][:, rows]
        ref = fx[nm]
        err = np.abs(got - ref).max()
        assert err <= 1e-5 * max(1.0, np.abs(ref).max()), (nm, err)
