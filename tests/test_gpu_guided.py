"""GPU parity of the guided uniform path (flash_attn_bsa_3d_variance_guided,
bsa_interface.py:1179-1260; flash_attn_bsa_3d_audio_guided, :1395-1501) through
the CUDA library.

* rho, the audio saliency, the Path B weights and the per-key-chunk scale are
  bit-exact against the CPU oracle (same operation order), which
  tests/test_oracle_guided.py pins to the reference's own values;
* Path B pooled keys match the reference's audio_weighted_mean_pooling_compression;
* the guided selection bitmaps are bit-exact against the oracle;
* outputs and gradients match the float64 oracle on that selection and the
  reference's fp32 outputs within max-abs 2e-2 and relative L2 1e-2;
* the unpadded dispatch with guidance equals the padded entry point.
"""
import numpy as np
import pytest
import torch

from helpers import bits, load_fixture, rel_l2
from inputs import GUIDED_CASES, make_inputs
from oracle import oracle as O
from prism_b200 import (_lib, audio_weighted_mean_pooling_compression,
                        compute_audio_spatial_concentration_gate, compute_block_audio_saliency,
                        compute_channel_variance_density, flash_attn_bsa_3d_audio_guided,
                        flash_attn_bsa_3d_variance_guided, ops, run_bsa_uniform)
from prism_b200.bsa_interface import build_uniform_plan
from prism_b200.guidance import guidance_inputs, make_guidance
from test_oracle_guided import guidance, select
from test_oracle_uniform import _setup, _tie_free_chunks

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref).max()
    r = rel_l2(got, ref)
    assert err <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {r:.3e}"


def _guidance_kw(case, inp, cuda):
    g = case.guidance
    if g["kind"] == "variance":
        return dict(variance_gamma=g["variance_gamma"])
    return dict(variance_gamma=g["variance_gamma"], audio_token_norms=inp["norms"].to(cuda),
                audio_gate=torch.tensor([g["gate"]], device=cuda), audio_gamma=g["audio_gamma"],
                audio_weighted_lambda=g["lambda_w"])


def _entry(case, inp, cuda):
    g = case.guidance
    gp = case.grid_padded
    kw = dict(sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
              chunk_3d_shape_q=case.chunk_q, chunk_3d_shape_k=case.chunk_k,
              valid_mask=None if inp["valid"] is None else inp["valid"].to(cuda))
    if g["kind"] == "variance":
        return lambda q, k, v: flash_attn_bsa_3d_variance_guided(
            q, k, v, gp, gp, variance_boost_gamma=g["variance_gamma"], **kw)
    norms = inp["norms"].to(cuda)
    gate = torch.tensor([g["gate"]], dtype=torch.bfloat16, device=cuda)
    gamma = torch.tensor(g["audio_gamma"], dtype=torch.bfloat16, device=cuda)
    return lambda q, k, v: flash_attn_bsa_3d_audio_guided(
        q, k, v, gp, gp, audio_token_norms=norms, audio_gate_value=gate, audio_boost_gamma=gamma,
        audio_weighted_lambda=g["lambda_w"], variance_boost_gamma=g["variance_gamma"], **kw)


def _plan(case, inp, cuda):
    gp = case.grid_padded
    valid = None if inp["valid"] is None else inp["valid"].to(cuda)
    plan = build_uniform_plan(gp, gp, case.chunk_q, case.chunk_k, case.head_dim, cuda,
                              sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                              valid_mask=valid)
    nk = plan.uniform["seq_k"] // plan.uniform["chunk_k"]
    plan.uniform["guidance"] = make_guidance(case.chunk_k, n_chunks_k=nk, device=cuda,
                                             **_guidance_kw(case, inp, cuda))
    q_re, k_re, v_re = (ops.gather_rows(inp[n][0].to(cuda), gp, gp,
                                        plan.src_idx if n == "q" else plan.src_idx_k)
                        for n in ("q", "k", "v"))
    return plan, q_re, k_re, v_re


@pytest.mark.parametrize("name", list(GUIDED_CASES))
def test_guidance_kernels_bit_exact(name, cuda):
    case = GUIDED_CASES[name]
    inp = make_inputs(case)
    r = _setup(name)
    ref = guidance(r)
    plan, q_re, k_re, v_re = _plan(case, inp, cuda)
    g = plan.uniform["guidance"]
    S, ck = r["S"], r["ck"]
    bits_k = plan.tile_bits
    fx = r["fx"]
    if ref["rho"] is not None:
        rho = ops.variance_density(v_re, S, case.chunk_k, bits_k).cpu().numpy()
        assert np.array_equal(rho.view(np.uint32), ref["rho"].view(np.uint32))
        np.testing.assert_allclose(rho, fx["rho"], rtol=2e-5, atol=1e-7)
    if g["norms"] is not None:
        a = ops.gather_values(g["norms"], plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
        from test_oracle_guided import norms_re
        assert np.array_equal(a.cpu().numpy()[:S], norms_re(r))
        sal = ops.audio_saliency(a, S, ck, bits_k).cpu().numpy()
        assert np.array_equal(sal.view(np.uint32), ref["saliency"].view(np.uint32))
        np.testing.assert_allclose(sal, fx["saliency"], rtol=2e-6, atol=1e-7)
        if ref["weights"] is not None:
            w = ops.audio_pool_weights(a, S, ck, bits_k, g["lambda_w"])
            assert np.array_equal(w.cpu().numpy().view(np.uint32), ref["weights"].view(np.uint32))
            kc = ops.pool_chunks(k_re, S, ck, weights=w).cpu().numpy()
            np.testing.assert_allclose(kc, fx["kcmp_pathb"], rtol=1e-5, atol=1e-6)
    weights, scale = guidance_inputs(plan, g, v_re)
    assert np.array_equal(scale.cpu().numpy().view(np.uint32), ref["scale"].view(np.uint32))
    assert (weights is None) == (ref["weights"] is None)


@pytest.mark.parametrize("name", list(GUIDED_CASES))
def test_guided_selection_bit_exact(name, cuda):
    case = GUIDED_CASES[name]
    inp = make_inputs(case)
    r = _setup(name)
    plan, q_re, k_re, v_re = _plan(case, inp, cuda)
    bq, bk = plan.select(q_re, k_re, v_re)
    rq, rk, sel = select(r, guidance(r))
    S = r["S"]
    nt, ntr = S // 64, q_re.shape[1] // 64
    gq = O.bits_to_dense(bq.cpu().numpy().view(np.uint32), ntr)
    gk = O.bits_to_dense(bk.cpu().numpy().view(np.uint32), ntr)
    assert np.array_equal(gq[:, :nt, :nt], O.bits_to_dense(rq, nt))
    assert np.array_equal(gk[:, :nt, :nt], O.bits_to_dense(rk, nt))
    assert not gq[:, nt:].any() and not gq[:, :, nt:].any()
    # and the reference's fp32 pass on the tie-free chunks (via the pinned oracle)
    ok = _tie_free_chunks(r)
    ref = O.bits_to_dense(r["fx"]["sel_chunks_f32"], S // r["ck"])
    assert (sel.astype(bool)[:, ok] == ref[:, ok]).all()


@pytest.mark.parametrize("name", list(GUIDED_CASES))
def test_guided_attention_parity(name, cuda):
    case = GUIDED_CASES[name]
    inp = make_inputs(case)
    r = _setup(name)
    fx = r["fx"]
    q, k, v = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    out = _entry(case, inp, cuda)(q, k, v)
    out.backward(inp["do"].to(cuda))
    assert _lib.load().prism_device_status() == 0
    got = {"o": out.detach()[0], "dq": q.grad[0], "dk": k.grad[0], "dv": v.grad[0]}
    got = {n: x.float().cpu().numpy() for n, x in got.items()}
    bq, _, _ = select(r, guidance(r))
    f = O.bf16_bits_to_f32
    src_q, src_k, inv_q, inv_k = r["src_q"], r["src_k"], r["inv_q"], r["inv_k"]
    qr, kr, vr = f(r["q"][:, src_q]), f(r["k"][:, src_k]), f(r["v"][:, src_k])
    o, _ = O.bsa_forward(qr, kr, vr, bq, r["valid_re"])
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, f(r["do"])[:, src_q], bq, r["valid_re"])
    ref = {"o": o[:, inv_q], "dq": dq[:, inv_q], "dk": dk[:, inv_k], "dv": dv[:, inv_k]}
    for n in ("o", "dq", "dk", "dv"):
        _close(got[n], ref[n], f"{n} vs oracle")
    ok_chunk = _tie_free_chunks(r)
    rows = fx["rows"]
    ok_rows = ok_chunk[inv_q[rows] // r["cq"]]
    for n in ("o", "dq"):
        _close(got[n][:, rows][:, ok_rows], fx[n][:, ok_rows], f"{n} vs reference")
    if ok_chunk.all():
        for n in ("dk", "dv"):
            _close(got[n][:, rows], fx[n], f"{n} vs reference")


@pytest.mark.parametrize("name", ["g_var_pad", "g_audio_pathb"])
def test_run_bsa_uniform_guided_fuses_padding(name, cuda):
    """The unpadded dispatch with guidance equals the padded guided entry point on
    the real tokens (norms zero-padded as wan_video_dit.py:301-306 does)."""
    case = GUIDED_CASES[name]
    inp = make_inputs(case)
    g = case.guidance
    gp = case.grid_padded
    qp, kp, vp = (inp[n].to(cuda) for n in ("q", "k", "v"))
    with torch.no_grad():
        outp = _entry(case, inp, cuda)(qp, kp, vp)
        qu, ku, vu = (inp[n + "_u"].to(cuda) for n in ("q", "k", "v"))
        kw = dict(sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                  chunk_3d_shape_q=case.chunk_q, chunk_3d_shape_k=case.chunk_k,
                  variance_boost_gamma=g.get("variance_gamma", 0.0))
        if g["kind"] == "audio":
            kw.update(audio_token_norms=inp["norms_u"].to(cuda),
                      audio_gate=torch.tensor([g["gate"]], device=cuda),
                      audio_boost_gamma=g["audio_gamma"], audio_weighted_lambda=g["lambda_w"])
        outu = run_bsa_uniform(qu, ku, vu, case.grid, **kw)
    T, H, W = case.grid
    h, D = case.heads, case.head_dim
    unpad = outp.view(1, h, *gp, D)[:, :, :T, :H, :W].reshape(1, h, T * H * W, D)
    assert torch.equal(outu, unpad)


@pytest.mark.parametrize("name", ["g_var_pad", "g_audio_pathb"])
def test_guidance_helpers(name, cuda):
    """The exported helpers on the reference's tensors (3D-chunk order, [1, H, S, D])."""
    case = GUIDED_CASES[name]
    inp = make_inputs(case)
    r = _setup(name)
    fx = r["fx"]
    S, ck = r["S"], r["ck"]
    tk, hk, wk = case.chunk_k
    src = torch.as_tensor(r["src_k"], device=cuda).long()
    vm = None if inp["valid"] is None else inp["valid"].to(cuda)[src]
    if "rho" in fx:
        v_ro = inp["v"].to(cuda)[:, :, src]
        rho = compute_channel_variance_density(v_ro, ck, tk, hk, wk, vm)
        np.testing.assert_allclose(rho.cpu().numpy(), fx["rho"], rtol=2e-5, atol=1e-7)
    if "saliency" in fx:
        a_ro = inp["norms"].to(cuda)[src]
        sal = compute_block_audio_saliency(a_ro, ck, valid_mask=vm)
        np.testing.assert_allclose(sal.cpu().numpy(), fx["saliency"], rtol=2e-6, atol=1e-7)
        if "kcmp_pathb" in fx:
            k_ro = inp["k"].to(cuda)[:, :, src]
            kc = audio_weighted_mean_pooling_compression(k_ro, ck, a_ro, valid_mask=vm,
                                                         lambda_w=case.guidance["lambda_w"])
            np.testing.assert_allclose(kc[0].cpu().numpy(), fx["kcmp_pathb"], rtol=1e-5, atol=1e-6)
        # the concentration gate: sigmoid(5 CV - 2) over the valid norms
        a = inp["norms"].float().numpy().astype(np.float64)
        m = np.ones_like(a, bool) if inp["valid"] is None else inp["valid"].numpy()
        mean = a[m].mean()
        cv = np.sqrt(((a[m] - mean) ** 2).mean()) / (mean + 1e-6)
        g = compute_audio_spatial_concentration_gate(inp["norms"].to(cuda), valid_mask=
                                                     None if inp["valid"] is None else inp["valid"].to(cuda))
        assert abs(float(g) - 1.0 / (1.0 + np.exp(-(5.0 * cv - 2.0)))) < 1e-5


def test_guided_errors(cuda):
    q = torch.zeros(2, 2, 512, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(NotImplementedError):
        flash_attn_bsa_3d_variance_guided(q, q, q, (8, 8, 8), (8, 8, 8))
    q1 = q[:1]
    with pytest.raises(NotImplementedError):
        flash_attn_bsa_3d_audio_guided(q1, q1, q1, (8, 8, 8), (8, 8, 8),
                                       score_modifier=torch.ones(3, device=cuda))
