"""GPU parity of cross-modal BSA (flash_attn_bsa_cross, bsa_interface.py:1276-1392):
query and key sequences of different lengths, 3D video and/or 1D audio sides.

* the chunk selection expanded to tiles is bit-exact against the CPU oracle
  (pinned to the reference by tests/test_oracle_cross.py);
* outputs and gradients match the float64 oracle on the same selection and the
  reference's fp32 outputs within max-abs 2e-2 and relative L2 1e-2;
* flash_attn_bsa_3d with latent_shape_q != latent_shape_k is the same computation.
"""
import numpy as np
import pytest
import torch

from helpers import bits, rel_l2
from inputs import CROSS_CASES, make_cross_inputs
from oracle import oracle as O
from prism_b200 import _lib, flash_attn_bsa_3d, flash_attn_bsa_cross, ops
from prism_b200.bsa_interface import build_cross_plan
from test_oracle_cross import chunk_bits, select, setup

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref).max()
    r = rel_l2(got, ref)
    assert err <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {r:.3e}"


def _kw(case):
    return dict(q_grid_size=case.q_shape if case.q_structure == "3d" else None,
                k_grid_size=case.k_shape if case.k_structure == "3d" else None,
                sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                chunk_size_q=case.chunk_size_q, chunk_size_k=case.chunk_size_k,
                chunk_3d_shape_q=case.chunk_3d_q, chunk_3d_shape_k=case.chunk_3d_k)


@pytest.mark.parametrize("name", list(CROSS_CASES))
def test_cross_selection_bit_exact(name, cuda):
    case = CROSS_CASES[name]
    inp = make_cross_inputs(case)
    plan = build_cross_plan(case.q_structure, case.k_structure, case.Sq, case.Sk, case.head_dim,
                            cuda, **_kw(case))
    q_re = ops.gather_rows(inp["q"][0].to(cuda), plan.grid, plan.grid_padded, plan.src_idx)
    k_re = ops.gather_rows(inp["k"][0].to(cuda), plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
    bq, bk = plan.select(q_re, k_re)
    r = setup(name)
    rq, rk, _ = select(r, want=False)
    nqt, nkt = r["q"]["Sp"] // 64, r["k"]["Sp"] // 64
    gq = O.bits_to_dense(bq.cpu().numpy().view(np.uint32), k_re.shape[1] // 64)
    gk = O.bits_to_dense(bk.cpu().numpy().view(np.uint32), q_re.shape[1] // 64)
    assert np.array_equal(gq[:, :nqt, :nkt], O.bits_to_dense(rq, nkt))
    assert np.array_equal(gk[:, :nkt, :nqt], O.bits_to_dense(rk, nqt))
    assert not gq[:, nqt:].any() and not gq[:, :, nkt:].any()
    # the gathers are the oracle's orders, zero rows past each side's grid
    assert np.array_equal(bits(q_re)[:, :r["q"]["Sp"]], r["q_re"])
    assert np.array_equal(bits(k_re)[:, :r["k"]["Sp"]], r["k_re"])


@pytest.mark.parametrize("name", list(CROSS_CASES))
def test_cross_attention_parity(name, cuda):
    case = CROSS_CASES[name]
    inp = make_cross_inputs(case)
    q, k, v = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    out = flash_attn_bsa_cross(q, k, v, case.q_structure, case.k_structure, **_kw(case))
    out.backward(inp["do"].to(cuda))
    assert _lib.load().prism_device_status() == 0
    assert out.shape == (1, case.heads, case.Sq, case.head_dim)
    got = {"o": out.detach()[0], "dq": q.grad[0], "dk": k.grad[0], "dv": v.grad[0]}
    got = {n: x.float().cpu().numpy() for n, x in got.items()}

    # float64 oracle on the oracle's selection (== the CUDA selection), every real row
    r = setup(name)
    bq, _, _ = select(r, want=False)
    f = O.bf16_bits_to_f32
    qr, kr, vr, dor = f(r["q_re"]), f(r["k_re"]), f(r["v_re"]), f(r["do_re"])
    o, _ = O.bsa_forward(qr, kr, vr, bq, r["k_valid"])
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, dor, bq, r["k_valid"])
    qrow = r["q"]["inv"][r["q"]["pidx"]]
    krow = r["k"]["inv"][r["k"]["pidx"]]
    ref = {"o": o[:, qrow], "dq": dq[:, qrow], "dk": dk[:, krow], "dv": dv[:, krow]}
    for n in ("o", "dq", "dk", "dv"):
        _close(got[n], ref[n], f"{n} vs oracle")
    # the reference's own fp32 outputs on its stored rows
    fx = r["fx"]
    for n, rows in (("o", fx["rows_q"]), ("dq", fx["rows_q"]), ("dk", fx["rows_k"]),
                    ("dv", fx["rows_k"])):
        _close(got[n][:, rows], fx[n], f"{n} vs reference")


def test_bsa_3d_different_latent_shapes(cuda):
    """flash_attn_bsa_3d with latent_shape_q != latent_shape_k (no padding) equals
    the cross path on the same grids."""
    case = CROSS_CASES["x_3d3d"]
    inp = make_cross_inputs(case)
    q, k, v = (inp[n].to(cuda) for n in ("q", "k", "v"))
    with torch.no_grad():
        a = flash_attn_bsa_cross(q, k, v, "3d", "3d", **_kw(case))
        b = flash_attn_bsa_3d(q, k, v, case.q_shape, case.k_shape, sparsity=case.sparsity,
                              cdf_threshold=case.cdf_threshold, chunk_3d_shape_q=case.chunk_3d_q,
                              chunk_3d_shape_k=case.chunk_3d_k)
    assert torch.equal(a, b)
