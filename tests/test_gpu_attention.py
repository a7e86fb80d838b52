"""GPU parity of the sparse attention kernels and of the full dynamic path.

Tolerance (from the task's north star): every bf16 output and gradient must
match within max-abs error 2e-2 and relative L2 error 1e-2 of the float64
oracle / the reference's fp32 outputs."""
import dataclasses
import math

import numpy as np
import pytest
import torch

from helpers import bits, load_fixture, rel_l2
from inputs import CASES, Case, make_inputs
from oracle import oracle as O
from prism_b200 import _lib, flash_attn_bsa_3d_dynamic, ops, run_bsa_dynamic

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref).max()
    r = rel_l2(got, ref)
    assert err <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {r:.3e}"


def _random_problem(heads, n_tiles, D, density, seed, dev, masked_tiles=(), empty_rows=()):
    g = torch.Generator().manual_seed(seed)
    S = n_tiles * 64
    q = torch.randn(heads, S, D, generator=g).to(torch.bfloat16)
    k = torch.randn(heads, S, D, generator=g).to(torch.bfloat16)
    v = torch.randn(heads, S, D, generator=g).to(torch.bfloat16)
    do = torch.randn(heads, S, D, generator=g).to(torch.bfloat16)
    sel = torch.rand(heads, n_tiles, n_tiles, generator=g) < density
    for r in empty_rows:
        sel[:, r, :] = False
    valid = torch.ones(S, dtype=torch.bool)
    tb = np.full(n_tiles, np.uint64(0xFFFFFFFFFFFFFFFF), dtype=np.uint64)
    for t, nvalid in masked_tiles:
        valid[t * 64 + nvalid:(t + 1) * 64] = False
        tb[t] = np.uint64((1 << nvalid) - 1) if nvalid < 64 else tb[t]
        if nvalid == 0:
            sel[:, :, t] = False  # fully padded key tiles are never selected
    bq = O.dense_to_bits(sel.numpy())
    bk = O.dense_to_bits(sel.numpy().transpose(0, 2, 1))
    dev_t = dict(q=q.to(dev), k=k.to(dev), v=v.to(dev), do=do.to(dev),
                 bq=torch.from_numpy(bq.view(np.int32)).to(dev),
                 bk=torch.from_numpy(bk.view(np.int32)).to(dev),
                 tb=torch.from_numpy(tb.view(np.int64)).to(dev))
    return dict(q=q, k=k, v=v, do=do, bq=bq, valid=valid.numpy(), dev=dev_t)


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("density", [0.3, 0.9])
def test_sparse_kernels_vs_oracle(D, density, cuda):
    pr = _random_problem(2, 16, D, density, seed=D + int(density * 10), dev=cuda,
                         masked_tiles=[(5, 17), (6, 0), (11, 63)], empty_rows=[3, 8, 9])
    d = pr["dev"]
    sm = 1.0 / math.sqrt(D)
    o, lse, o_lo = ops.bsa_fwd(d["q"], d["k"], d["v"], d["bq"], d["tb"], sm, want_lo=True)
    f = lambda t: t.float().numpy()
    ro, rlse = O.bsa_forward(f(pr["q"]), f(pr["k"]), f(pr["v"]), pr["bq"], pr["valid"], sm)
    _close(o.float().cpu(), ro, "O")
    l = lse.cpu().numpy()
    fin = np.isfinite(rlse)
    assert np.array_equal(np.isfinite(l), fin)
    assert np.abs(l[fin] - rlse[fin]).max() < 1e-2
    # o + o_lo is the fp32 accumulator result (limited by the bf16 P of the PV
    # product, not by the bf16 rounding of O)
    hi_lo = (o.float() + o_lo.float()).cpu().numpy()
    assert np.abs(hi_lo - ro).max() < 5e-3
    dq, dk, dv = ops.bsa_bwd(d["q"], d["k"], d["v"], o, d["do"], lse, d["bq"], d["bk"], d["tb"], sm,
                             o_lo=o_lo)
    rdq, rdk, rdv = O.bsa_backward(f(pr["q"]), f(pr["k"]), f(pr["v"]), ro, f(pr["do"]), pr["bq"],
                                   pr["valid"], sm)
    _close(dq.float().cpu(), rdq, "dQ")
    _close(dk.float().cpu(), rdk, "dK")
    _close(dv.float().cpu(), rdv, "dV")
    # empty rows: O = 0, lse = -inf, dQ = 0
    for r in (3, 8, 9):
        assert (o[:, r * 64:(r + 1) * 64] == 0).all()
        assert torch.isinf(lse[:, r * 64:(r + 1) * 64]).all()
        assert (dq[:, r * 64:(r + 1) * 64] == 0).all()
    # determinism
    o2, _ = ops.bsa_fwd(d["q"], d["k"], d["v"], d["bq"], d["tb"], sm)
    assert torch.equal(o, o2)
    dq2, dk2, dv2 = ops.bsa_bwd(d["q"], d["k"], d["v"], o, d["do"], lse, d["bq"], d["bk"], d["tb"], sm,
                                o_lo=o_lo)
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)
    assert _lib.load().prism_device_status() == 0, "a bounded wait inside a kernel gave up"


@pytest.mark.parametrize("D", [64, 128])
def test_sparse_kernels_multiword_rows(D, cuda):
    """72 tiles per head (3 bitmap words per row), half density with padded
    and fully padded key tiles: exercises the K/V and Q/dO rings wrapping many
    times, odd tile counts in the forward's tile pairs, and word boundaries."""
    pr = _random_problem(2, 72, D, 0.5, seed=7 + D, dev=cuda,
                         masked_tiles=[(0, 40), (31, 1), (32, 0), (63, 64), (71, 33)],
                         empty_rows=[10, 57])
    d = pr["dev"]
    sm = 1.0 / math.sqrt(D)
    o, lse, o_lo = ops.bsa_fwd(d["q"], d["k"], d["v"], d["bq"], d["tb"], sm, want_lo=True)
    f = lambda t: t.float().numpy()
    ro, _ = O.bsa_forward(f(pr["q"]), f(pr["k"]), f(pr["v"]), pr["bq"], pr["valid"], sm)
    _close(o.float().cpu(), ro, "O")
    dq, dk, dv = ops.bsa_bwd(d["q"], d["k"], d["v"], o, d["do"], lse, d["bq"], d["bk"], d["tb"], sm,
                             o_lo=o_lo)
    rdq, rdk, rdv = O.bsa_backward(f(pr["q"]), f(pr["k"]), f(pr["v"]), ro, f(pr["do"]), pr["bq"],
                                   pr["valid"], sm)
    _close(dq.float().cpu(), rdq, "dQ")
    _close(dk.float().cpu(), rdk, "dK")
    _close(dv.float().cpu(), rdv, "dV")
    assert _lib.load().prism_device_status() == 0, "a bounded wait inside a kernel gave up"


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("density", [0.08, 0.5])
def test_sparse_kernels_odd_tile_pairs(D, density, cuda):
    """S % 256 == 128: the last forward CTA holds a single group of 128 rows;
    low densities make most key tiles selected by one group only."""
    pr = _random_problem(2, 18, D, density, seed=7 * D + int(density * 100), dev=cuda,
                         masked_tiles=[(17, 20), (3, 0)], empty_rows=[16])
    d = pr["dev"]
    sm = 1.0 / math.sqrt(D)
    o, lse, o_lo = ops.bsa_fwd(d["q"], d["k"], d["v"], d["bq"], d["tb"], sm, want_lo=True)
    f = lambda t: t.float().numpy()
    ro, rlse = O.bsa_forward(f(pr["q"]), f(pr["k"]), f(pr["v"]), pr["bq"], pr["valid"], sm)
    _close(o.float().cpu(), ro, "O")
    dq, dk, dv = ops.bsa_bwd(d["q"], d["k"], d["v"], o, d["do"], lse, d["bq"], d["bk"], d["tb"], sm,
                             o_lo=o_lo)
    rdq, rdk, rdv = O.bsa_backward(f(pr["q"]), f(pr["k"]), f(pr["v"]), ro, f(pr["do"]), pr["bq"],
                                   pr["valid"], sm)
    _close(dq.float().cpu(), rdq, "dQ")
    _close(dk.float().cpu(), rdk, "dK")
    _close(dv.float().cpu(), rdv, "dV")
    assert (o[:, 16 * 64:17 * 64] == 0).all()
    assert _lib.load().prism_device_status() == 0, "a bounded wait inside a kernel gave up"


@pytest.mark.parametrize("name", [n for n, c in CASES.items() if c.needs_pad])
def test_dynamic_path_vs_reference_golden(name, cuda):
    """flash_attn_bsa_3d_dynamic (reference signature, padded THW input) against
    the reference's own fp32 outputs and gradients stored in the fixture."""
    case = CASES[name]
    fx = load_fixture(name)
    inp = make_inputs(case)
    q, k, v = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    out, ids = flash_attn_bsa_3d_dynamic(
        q, k, v, case.grid_padded, method=case.method, sparsity=case.sparsity,
        cdf_threshold=case.cdf_threshold,
        audio_token_norms=None if inp["norms"] is None else inp["norms"].to(cuda),
        valid_mask=inp["valid"].to(cuda), lambda_a=case.lambda_a, tau_128=case.tau_128,
        lambda_128=case.lambda_128, return_shape_ids=True)
    assert np.array_equal(ids.cpu().numpy(), fx["shape_ids"])
    out.backward(inp["do"].to(cuda))
    rows = fx["rows"]
    # padding rows of O depend on the reference's topk tie order (all scores tie there)
    real = inp["valid"].numpy()[rows]
    _close(out.detach()[0].float().cpu().numpy()[:, rows][:, real], fx["o"][:, real], "O")
    _close(q.grad[0].float().cpu().numpy()[:, rows], fx["dq"], "dQ")
    _close(k.grad[0].float().cpu().numpy()[:, rows], fx["dk"], "dK")
    _close(v.grad[0].float().cpu().numpy()[:, rows], fx["dv"], "dV")
    # cached shape ids reproduce the same output bit for bit (checkpoint recompute)
    with torch.no_grad():
        out2 = flash_attn_bsa_3d_dynamic(
            q, k, v, case.grid_padded, method=case.method, sparsity=case.sparsity,
            cdf_threshold=case.cdf_threshold, valid_mask=inp["valid"].to(cuda), shape_ids=ids)
    assert torch.equal(out.detach(), out2)


@pytest.mark.parametrize("D", [16, 32])
def test_dynamic_path_small_head_dim(D, cuda):
    """Head dims 16 and 32 (accepted by the reference, bsa_interface.py:604-605) through
    flash_attn_bsa_3d_dynamic: shape ids bit-exact against the oracle; output and the
    three gradients within the tolerance of the float64 oracle on the oracle's selection."""
    case = dataclasses.replace(CASES["mixed_d64"], head_dim=D, name=f"mixed_d{D}")
    inp = make_inputs(case)
    q, k, v = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    out, ids = flash_attn_bsa_3d_dynamic(
        q, k, v, case.grid_padded, method=case.method, sparsity=case.sparsity,
        cdf_threshold=case.cdf_threshold, audio_token_norms=inp["norms"].to(cuda),
        valid_mask=inp["valid"].to(cuda), lambda_a=case.lambda_a, tau_128=case.tau_128,
        lambda_128=case.lambda_128, return_shape_ids=True)
    out.backward(inp["do"].to(cuda))
    b16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    r = O.dynamic_forward_selection(b16(inp["q"][0]), b16(inp["k"][0]), b16(inp["v"][0]),
                                    case.grid_padded, method=case.method, sparsity=case.sparsity,
                                    cdf_threshold=case.cdf_threshold, norms_bits=b16(inp["norms"]),
                                    valid=inp["valid"].numpy().astype(np.uint8), lambda_a=case.lambda_a,
                                    tau_128=case.tau_128, lambda_128=case.lambda_128)
    assert np.array_equal(ids.cpu().numpy(), r["shape_ids"])
    f = O.bf16_bits_to_f32
    qr, kr, vr = f(r["q_re"]), f(r["k_re"]), f(r["v_re"])
    o, _ = O.bsa_forward(qr, kr, vr, r["bits_q"], r["valid_re"])
    do_re = inp["do"][0].float().numpy()[:, r["src_idx"]]
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, do_re, r["bits_q"], r["valid_re"])
    inv = r["inv_idx"]
    for name, got, ref in (("O", out.detach()[0], o), ("dQ", q.grad[0], dq), ("dK", k.grad[0], dk),
                           ("dV", v.grad[0], dv)):
        _close(got.float().cpu().numpy(), ref[:, inv], f"{name} (D={D})")
    assert _lib.load().prism_device_status() == 0, "a bounded wait inside a kernel gave up"


@pytest.mark.parametrize("layout", ["bhsd", "bshd"])
def test_run_bsa_dynamic_fuses_padding(layout, cuda):
    """The unpadded entry point equals the padded one on the real tokens, for
    the output and for all three gradients."""
    case = CASES["mixed_d128_penalty"]
    inp = make_inputs(case)
    kw = dict(method=case.method, sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
              lambda_a=case.lambda_a, tau_128=case.tau_128, lambda_128=case.lambda_128)
    qp, kp, vp = (inp[n].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    outp = flash_attn_bsa_3d_dynamic(qp, kp, vp, case.grid_padded,
                                     audio_token_norms=inp["norms"].to(cuda),
                                     valid_mask=inp["valid"].to(cuda), **kw)
    outp.backward(inp["do"].to(cuda))
    T, H, W = case.grid
    Tp, Hp, Wp = case.grid_padded
    h, D = case.heads, case.head_dim

    def unpad(x):
        return x.detach().view(1, h, Tp, Hp, Wp, D)[:, :, :T, :H, :W].reshape(1, h, T * H * W, D)

    qu, ku, vu, dou = (inp[n + "_u"].to(cuda) for n in ("q", "k", "v", "do"))
    if layout == "bshd":
        qu, ku, vu, dou = (x.transpose(1, 2).contiguous() for x in (qu, ku, vu, dou))
    qu, ku, vu = (x.requires_grad_(True) for x in (qu, ku, vu))
    outu = run_bsa_dynamic(qu, ku, vu, case.grid, audio_token_norms=inp["norms_u"].to(cuda),
                           layout=layout, **kw)
    outu.backward(dou)
    tr = (lambda x: x.transpose(1, 2)) if layout == "bshd" else (lambda x: x)
    assert torch.equal(tr(outu.detach()), unpad(outp))
    for gu, gp in ((qu.grad, qp.grad), (ku.grad, kp.grad), (vu.grad, vp.grad)):
        assert torch.equal(tr(gu), unpad(gp))


def test_c1_scale_sampled(cuda):
    """Config-1 grid (21x45x80 -> 24x48x80, D=128) on 2 heads: selection is
    deterministic and sampled q tiles match a float64 per-tile recomputation."""
    case = Case("c1x2", (21, 45, 80), 2, 128, values="zoned", sparsity=0.92, cdf_threshold=0.9,
                audio_tokens=64, seed=0)
    inp = make_inputs(case)
    qu, ku, vu = (inp[n + "_u"].to(cuda) for n in ("q", "k", "v"))
    out, plan = run_bsa_dynamic(qu, ku, vu, case.grid, audio_token_norms=inp["norms_u"].to(cuda),
                                sparsity=0.92, cdf_threshold=0.9, return_plan=True)
    bq1 = plan.bits_q.clone()
    out2, plan2 = run_bsa_dynamic(qu, ku, vu, case.grid, audio_token_norms=inp["norms_u"].to(cuda),
                                  sparsity=0.92, cdf_threshold=0.9, return_plan=True)
    assert torch.equal(bq1, plan2.bits_q) and torch.equal(out, out2)
    gp = case.grid_padded
    src = plan.src_idx.cpu().numpy()
    inv = plan.inv_idx.cpu().numpy()
    nt = src.size // 64
    dense = O.bits_to_dense(plan.bits_q.cpu().numpy().view(np.uint32), nt)
    tb = plan.tile_bits.cpu().numpy().view(np.uint64)
    T, H, W = case.grid
    Tp, Hp, Wp = gp
    qp = inp["q"][0].float().numpy()[:, src]
    kp = inp["k"][0].float().numpy()[:, src]
    vp = inp["v"][0].float().numpy()[:, src]
    o_pad = np.zeros((2, Tp * Hp * Wp, 128))
    o_pad.reshape(2, Tp, Hp, Wp, 128)[:, :T, :H, :W] = out[0].float().cpu().numpy().reshape(2, T, H, W, 128)
    o_re = o_pad[:, src]
    rng = np.random.default_rng(0)
    for h in range(2):
        for qt in rng.choice(nt, 6, replace=False):
            cols = np.nonzero(dense[h, qt])[0]
            keys = (cols[:, None] * 64 + np.arange(64)[None]).reshape(-1)
            kvalid = np.unpackbits(tb[cols].view(np.uint8), bitorder="little").astype(bool)
            rows = np.arange(qt * 64, qt * 64 + 64)
            s = qp[h, rows] @ kp[h, keys].T / math.sqrt(128)
            s[:, ~kvalid] = -np.inf
            p = np.exp(s - s.max(1, keepdims=True))
            ref = (p / p.sum(1, keepdims=True)) @ vp[h, keys]
            real = np.array([(src[r] // (Hp * Wp) < T) and ((src[r] // Wp) % Hp < H) and (src[r] % Wp < W) for r in rows])
            if real.any():
                _close(o_re[h, rows][real], ref[real], f"head {h} tile {qt}")
