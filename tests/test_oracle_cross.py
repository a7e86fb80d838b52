"""Pin the CPU oracle's cross-modal path (different query and key lengths)
against golden vectors produced by the reference's own ``flash_attn_bsa_cross``
(bsa_interface.py:1276-1392, run on CPU by tests/golden/make_golden.py).

Each side is "3d" (a latent grid padded per axis to its chunk) or "1d" (a token
sequence padded to its chunk).  A padded q side pools q over its real rows, a
padded k side masks its padding keys (bsa_interface.py:606-611).

* the chunk-level selection equals the reference's fp32 pass (the oracle, like
  the CUDA path, pools and scores in fp32);
* on the selection the reference made, the float64 attention restatement agrees
  with the reference's fp32 Triton kernels to ~1e-5.
"""
import math

import numpy as np
import pytest

from helpers import load_fixture
from inputs import CROSS_CASES, make_cross_inputs
from oracle import oracle as O


def _b(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def side_layout(structure, shape, chunk_1d, chunk_3d):
    """(grid, padded grid, chunk) of one side, 1D sides as (1, 1, S) grids."""
    if structure == "3d":
        chunk = tuple(chunk_3d or (4, 4, 4))
        grid = tuple(shape)
        return grid, tuple(int(math.ceil(g / c) * c) for g, c in zip(grid, chunk)), chunk
    (S,) = shape
    return (1, 1, S), (1, 1, int(math.ceil(S / chunk_1d) * chunk_1d)), (1, 1, chunk_1d)


def padded_index(grid, gp):
    """Padded THW index of every real token (real tokens in THW order)."""
    T, H, W = grid
    t, h, w = np.meshgrid(np.arange(T), np.arange(H), np.arange(W), indexing="ij")
    return ((t * gp[1] + h) * gp[2] + w).reshape(-1)


def setup(name):
    case = CROSS_CASES[name]
    inp = make_cross_inputs(case)
    r = dict(case=case, fx=load_fixture(name))
    for side, st, shape, c1, c3 in (("q", case.q_structure, case.q_shape, case.chunk_size_q,
                                     case.chunk_3d_q),
                                    ("k", case.k_structure, case.k_shape, case.chunk_size_k,
                                     case.chunk_3d_k)):
        grid, gp, chunk = side_layout(st, shape, c1, c3)
        Sp = gp[0] * gp[1] * gp[2]
        src, inv = O.uniform_layout(gp, chunk)
        pidx = padded_index(grid, gp)
        valid = np.zeros(Sp, bool)
        valid[pidx] = True
        r[side] = dict(grid=grid, gp=gp, chunk=int(np.prod(chunk)), Sp=Sp, src=src, inv=inv,
                       pidx=pidx, padded=grid != gp, valid_re=valid[src])
    for nm, side in (("q", "q"), ("k", "k"), ("v", "k"), ("do", "q")):
        x = _b(inp[nm][0])  # [h, S, D] real tokens
        s = r[side]
        full = np.zeros((x.shape[0], s["Sp"], x.shape[2]), np.uint16)
        full[:, s["pidx"]] = x
        r[nm + "_re"] = full[:, s["src"]]
    # rows the q pooling counts: q's own mask if q is padded, else the key mask when
    # the lengths agree, else every row (bsa_interface.py:606-611)
    if r["q"]["padded"]:
        r["q_pool"] = r["q"]["valid_re"]
    elif r["k"]["padded"] and r["q"]["Sp"] == r["k"]["Sp"]:
        r["q_pool"] = r["k"]["valid_re"]
    else:
        r["q_pool"] = None
    r["k_valid"] = r["k"]["valid_re"] if r["k"]["padded"] else None
    return r


def select(r, want=True):
    case = r["case"]
    return O.block_select_uniform(r["q_re"], r["k_re"], r["q"]["Sp"], r["k"]["Sp"], r["q"]["chunk"],
                                  r["k"]["chunk"], r["q_pool"], r["k_valid"], case.sparsity,
                                  case.cdf_threshold, want_chunks=want)


def chunk_bits(sel, r):
    """Chunk selection [h, nq, nk] -> tile bitmap (tiles without a valid key dropped)."""
    tq, tk = r["q"]["chunk"] // 64, r["k"]["chunk"] // 64
    exp = np.repeat(np.repeat(sel.astype(bool), tq, axis=1), tk, axis=2)
    if r["k_valid"] is not None:
        exp &= r["k_valid"].reshape(-1, 64).any(axis=1)[None, None, :]
    return O.dense_to_bits(exp)


@pytest.mark.parametrize("name", list(CROSS_CASES))
def test_cross_selection_matches_reference(name):
    r = setup(name)
    bits_q, bits_k, sel = select(r)
    nk = r["k"]["Sp"] // r["k"]["chunk"]
    ref = O.bits_to_dense(r["fx"]["sel_chunks_f32"], nk)
    assert (sel.astype(bool) == ref).all(), f"{(sel.astype(bool) != ref).sum()} chunk pairs differ"
    assert (bits_q == chunk_bits(sel, r)).all()
    nqt, nkt = r["q"]["Sp"] // 64, r["k"]["Sp"] // 64
    assert (O.bits_to_dense(bits_k, nqt) == O.bits_to_dense(bits_q, nkt).transpose(0, 2, 1)).all()


@pytest.mark.parametrize("name", list(CROSS_CASES))
def test_cross_attention_restatement(name):
    r = setup(name)
    nk = r["k"]["Sp"] // r["k"]["chunk"]
    bq = chunk_bits(O.bits_to_dense(r["fx"]["sel_chunks_f32"], nk), r)
    f = O.bf16_bits_to_f32
    qr, kr, vr, dor = f(r["q_re"]), f(r["k_re"]), f(r["v_re"]), f(r["do_re"])
    o, _ = O.bsa_forward(qr, kr, vr, bq, r["k_valid"])
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, dor, bq, r["k_valid"])
    fx = r["fx"]
    qrow = r["q"]["inv"][r["q"]["pidx"]]  # real query token -> row of the q order
    krow = r["k"]["inv"][r["k"]["pidx"]]
    for nm, x, rows, side in (("o", o, fx["rows_q"], qrow), ("dq", dq, fx["rows_q"], qrow),
                              ("dk", dk, fx["rows_k"], krow), ("dv", dv, fx["rows_k"], krow)):
        got = x[:, side[rows]]
        ref = fx[nm]
        err = np.abs(got - ref).max()
        assert err <= 1e-5 * max(1.0, np.abs(ref).max()), (nm, err)
