"""GPU parity of the uniform fixed-shape path (flash_attn_bsa_3d,
bsa_interface.py:1123-1176) through the CUDA library.

* chunk orders and selection bitmaps are bit-exact against the CPU oracle
  (which tests/test_oracle_uniform.py pins to the reference's own outputs);
* outputs and gradients match the float64 oracle on the same selection, and the
  reference's fp32 outputs stored in the fixtures, within max-abs 2e-2 and
  relative L2 1e-2 (bf16 inputs and outputs);
* the unpadded entry point equals the padded one bit for bit.
"""
import numpy as np
import pytest
import torch

from helpers import bits, load_fixture, rel_l2
from inputs import UNIFORM_CASES, make_inputs
from oracle import oracle as O
from prism_b200 import _lib, flash_attn_bsa_3d, ops, run_bsa_uniform

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref).max()
    r = rel_l2(got, ref)
    assert err <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {r:.3e}"


def _vol(c):
    return int(c[0] * c[1] * c[2])


@pytest.mark.parametrize("name", list(UNIFORM_CASES))
def test_uniform_layout_kernel(name, cuda):
    case = UNIFORM_CASES[name]
    gp = case.grid_padded
    S = gp[0] * gp[1] * gp[2]
    n_rows = -(-S // 128) * 128
    for chunk in (case.chunk_q, case.chunk_k):
        src, inv = ops.uniform_layout(gp, chunk, n_rows, cuda)
        rsrc, rinv = O.uniform_layout(gp, chunk, n_rows)
        assert np.array_equal(src.cpu().numpy(), rsrc)
        assert np.array_equal(inv.cpu().numpy(), rinv)


def _plan_and_gather(case, inp, cuda):
    from prism_b200.bsa_interface import build_uniform_plan
    gp = case.grid_padded
    D = case.head_dim
    valid = None if inp["valid"] is None else inp["valid"].to(cuda)
    plan = build_uniform_plan(gp, gp, case.chunk_q, case.chunk_k, D, cuda,
                              sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                              valid_mask=valid)
    q_re = ops.gather_rows(inp["q"][0].to(cuda), gp, gp, plan.src_idx)
    k_re = ops.gather_rows(inp["k"][0].to(cuda), gp, gp, plan.src_idx_k)
    return plan, q_re, k_re


@pytest.mark.parametrize("name", list(UNIFORM_CASES))
def test_uniform_selection_bit_exact(name, cuda):
    case = UNIFORM_CASES[name]
    inp = make_inputs(case)
    plan, q_re, k_re = _plan_and_gather(case, inp, cuda)
    seq = plan.uniform["seq_q"]
    n_rows = q_re.shape[1]
    # the gather is the oracle's permutation, with zero rows past the grid
    src_q = plan.src_idx.cpu().numpy()
    qb = bits(inp["q"][0])
    assert np.array_equal(bits(q_re)[:, :seq], qb[:, src_q[:seq]])
    assert not bits(q_re)[:, seq:].any()
    bq, bk = plan.select(q_re, k_re)
    src_k = plan.src_idx_k.cpu().numpy()[:seq]
    valid_re = None if inp["valid"] is None else inp["valid"].numpy()[src_k]
    rq, rk, _ = O.block_select_uniform(qb[:, src_q[:seq]], bits(inp["k"][0])[:, src_k], seq, seq,
                                       plan.uniform["chunk_q"], plan.uniform["chunk_k"], valid_re,
                                       valid_re, case.sparsity, case.cdf_threshold)
    nt, ntr = seq // 64, n_rows // 64
    gq = O.bits_to_dense(bq.cpu().numpy().view(np.uint32), ntr)
    gk = O.bits_to_dense(bk.cpu().numpy().view(np.uint32), ntr)
    assert np.array_equal(gq[:, :nt, :nt], O.bits_to_dense(rq, nt))
    assert np.array_equal(gk[:, :nt, :nt], O.bits_to_dense(rk, nt))
    assert not gq[:, nt:].any() and not gq[:, :, nt:].any()
    # key validity of the padding tiles is empty
    tb = plan.tile_bits.cpu().numpy()
    assert not tb[nt:].any()


@pytest.mark.parametrize("name", list(UNIFORM_CASES))
def test_flash_attn_bsa_3d_parity(name, cuda):
    """Reference signature on the padded grid: against the float64 oracle on the
    same selection (every row), and against the reference's fp32 outputs on
    rows that do not depend on torch.topk's tie order."""
    case = UNIFORM_CASES[name]
    fx = load_fixture(name)
    inp = make_inputs(case)
    gp = case.grid_padded
    S = gp[0] * gp[1] * gp[2]
    q, k, v = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    valid = None if inp["valid"] is None else inp["valid"].to(cuda)
    out = flash_attn_bsa_3d(q, k, v, gp, gp, sparsity=case.sparsity,
                            cdf_threshold=case.cdf_threshold, chunk_3d_shape_q=case.chunk_q,
                            chunk_3d_shape_k=case.chunk_k, valid_mask=valid)
    out.backward(inp["do"].to(cuda))
    assert _lib.load().prism_device_status() == 0
    got = {"o": out.detach()[0], "dq": q.grad[0], "dk": k.grad[0], "dv": v.grad[0]}
    got = {n: x.float().cpu().numpy() for n, x in got.items()}

    # float64 oracle on the oracle's own selection (== the CUDA selection)
    src_q, inv_q = O.uniform_layout(gp, case.chunk_q)
    src_k, inv_k = O.uniform_layout(gp, case.chunk_k)
    valid_re = None if inp["valid"] is None else inp["valid"].numpy()[src_k]
    f = O.bf16_bits_to_f32
    qb, kb, vb, dob = (bits(inp[n][0]) for n in ("q", "k", "v", "do"))
    bq, _, _ = O.block_select_uniform(qb[:, src_q], kb[:, src_k], S, S, _vol(case.chunk_q),
                                      _vol(case.chunk_k), valid_re, valid_re, case.sparsity,
                                      case.cdf_threshold)
    qr, kr, vr = f(qb[:, src_q]), f(kb[:, src_k]), f(vb[:, src_k])
    o, _ = O.bsa_forward(qr, kr, vr, bq, valid_re)
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, f(dob)[:, src_q], bq, valid_re)
    ref = {"o": o[:, inv_q], "dq": dq[:, inv_q], "dk": dk[:, inv_k], "dv": dv[:, inv_k]}
    for n in ("o", "dq", "dk", "dv"):
        _close(got[n], ref[n], f"{n} vs oracle")

    # reference fp32 outputs: rows whose q chunk has a row valid under the
    # key-order mask (the others tie on every score); dK / dV sum over all q
    # rows, so they are compared only when no q chunk ties
    rows = fx["rows"]
    cq = _vol(case.chunk_q)
    if valid_re is None:
        ok_chunk = np.ones(S // cq, bool)
    else:
        ok_chunk = valid_re.reshape(S // cq, cq).any(axis=1)
    ok_rows = ok_chunk[inv_q[rows] // cq]
    for n in ("o", "dq"):
        _close(got[n][:, rows][:, ok_rows], fx[n][:, ok_rows], f"{n} vs reference")
    if ok_chunk.all():
        for n in ("dk", "dv"):
            _close(got[n][:, rows], fx[n], f"{n} vs reference")


@pytest.mark.parametrize("layout", ["bhsd", "bshd"])
@pytest.mark.parametrize("name", ["u64_pad", "umix_cdf"])
def test_run_bsa_uniform_fuses_padding(name, layout, cuda):
    """The unpadded entry point equals flash_attn_bsa_3d on the padded grid, on
    the real tokens, for the output and all three gradients."""
    case = UNIFORM_CASES[name]
    inp = make_inputs(case)
    gp = case.grid_padded
    kw = dict(sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
              chunk_3d_shape_q=case.chunk_q, chunk_3d_shape_k=case.chunk_k)
    qp, kp, vp = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    outp = flash_attn_bsa_3d(qp, kp, vp, gp, gp, valid_mask=inp["valid"].to(cuda), **kw)
    outp.backward(inp["do"].to(cuda))
    T, H, W = case.grid
    Tp, Hp, Wp = gp
    h, D = case.heads, case.head_dim

    def unpad(x):
        return x.detach().view(1, h, Tp, Hp, Wp, D)[:, :, :T, :H, :W].reshape(1, h, T * H * W, D)

    qu, ku, vu, dou = (inp[n + "_u"].to(cuda) for n in ("q", "k", "v", "do"))
    if layout == "bshd":
        qu, ku, vu, dou = (x.transpose(1, 2).contiguous() for x in (qu, ku, vu, dou))
    qu, ku, vu = (x.requires_grad_(True) for x in (qu, ku, vu))
    outu = run_bsa_uniform(qu, ku, vu, case.grid, layout=layout, **kw)
    outu.backward(dou)
    tr = (lambda x: x.transpose(1, 2)) if layout == "bshd" else (lambda x: x)
    assert torch.equal(tr(outu.detach()), unpad(outp))
    for gu, gpd in ((qu.grad, qp.grad), (ku.grad, kp.grad), (vu.grad, vp.grad)):
        assert torch.equal(tr(gu), unpad(gpd))


def test_uniform_batch_folds_into_heads(cuda):
    """B > 1: each batch entry is attended independently (as the reference's
    kernels index (batch, head) pairs)."""
    case = UNIFORM_CASES["u64_pad"]
    inp = make_inputs(case)
    gp = case.grid_padded
    kw = dict(sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
              chunk_3d_shape_q=case.chunk_q, chunk_3d_shape_k=case.chunk_k,
              valid_mask=inp["valid"].to(cuda))
    q, k, v = (inp[n].to(cuda) for n in ("q", "k", "v"))
    with torch.no_grad():
        one = flash_attn_bsa_3d(q, k, v, gp, gp, **kw)
        two = flash_attn_bsa_3d(torch.cat([q, q.flip(1)]), torch.cat([k, k.flip(1)]),
                                torch.cat([v, v.flip(1)]), gp, gp, **kw)
    assert torch.equal(two[0:1], one)
    assert torch.equal(two[1:2], one.flip(1))


def test_uniform_errors(cuda):
    q = torch.zeros(1, 2, 512, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        flash_attn_bsa_3d(q, q, q, (8, 8, 8), (8, 8, 8), sparsity=None, cdf_threshold=None)
    with pytest.raises(NotImplementedError):
        flash_attn_bsa_3d(q, q, q, (8, 8, 8), (8, 8, 8), chunk_3d_shape_q=(2, 4, 4),
                          chunk_3d_shape_k=(2, 4, 4))
    with pytest.raises(AssertionError):
        flash_attn_bsa_3d(q, q, q, (8, 8, 8), (8, 8, 8), chunk_3d_shape_q=(3, 4, 4))


@pytest.mark.parametrize("sparsity,cdf", [(0.95, 0.45), (0.9, 0.3), (0.5, 0.1), (0.75, 0.49)])
def test_selection_paths_bit_exact(sparsity, cdf, cuda):
    """Hybrid top-k + cumulative-mass selection on flat random scores (N(0, 1) rows
    pooled over 64 tokens), where the top-k chunks often hold less than the mass
    threshold: both the top-k-first shortcut and its fallback to the mass passes run,
    and the bitmaps equal the oracle's."""
    g = torch.Generator().manual_seed(int(sparsity * 100 + cdf * 1000))
    heads, D, S = 2, 64, 64 * 96
    q = torch.randn(heads, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(heads, S, D, generator=g).to(torch.bfloat16)
    bits_k = torch.full((S // 64,), -1, dtype=torch.int64)  # every key valid
    bq, bk = ops.block_select_uniform(q.to(cuda), k.to(cuda), S, S, 64, 64, None, bits_k.to(cuda),
                                      sparsity, cdf)
    rq, rk, _ = O.block_select_uniform(bits(q), bits(k), S, S, 64, 64, None, None, sparsity, cdf)
    n = S // 64
    assert np.array_equal(O.bits_to_dense(bq.cpu().numpy().view(np.uint32), n), O.bits_to_dense(rq, n))
    assert np.array_equal(O.bits_to_dense(bk.cpu().numpy().view(np.uint32), n), O.bits_to_dense(rk, n))
