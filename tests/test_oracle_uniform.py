"""Pin the CPU oracle's uniform fixed-shape path against golden vectors produced
by the reference's own ``flash_attn_bsa_3d`` (bsa_interface.py:1123-1176, run
on CPU by tests/golden/make_golden.py).

* the 3D-chunk orders (rearrange_THW_to_3d_block) are identical;
* the chunk-level selection is identical, except for a q chunk whose rows are
  all masked under the key-order mask the reference applies to q
  (bsa_interface.py:609-610): its pooled q is 0, every score ties, and the
  reference's choice among them is torch.topk's unspecified tie order;
* on the selection the reference made, the float64 attention restatement
  agrees with the reference's fp32 Triton kernels (run under TRITON_INTERPRET)
  to ~1e-5 on every stored row.
"""
import numpy as np
import pytest

from helpers import load_fixture
from inputs import UNIFORM_CASES, UNIFORM_CASES_ALL, make_inputs
from oracle import oracle as O


def _b(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _setup(name):
    case = UNIFORM_CASES_ALL[name]
    fx = load_fixture(name)
    inp = make_inputs(case)
    gp = case.grid_padded
    S = gp[0] * gp[1] * gp[2]
    src_q, inv_q = O.uniform_layout(gp, case.chunk_q)
    src_k, inv_k = O.uniform_layout(gp, case.chunk_k)
    q, k, v, do = (_b(inp[n][0]) for n in ("q", "k", "v", "do"))
    valid = None if inp["valid"] is None else inp["valid"].numpy().astype(bool)
    valid_re = None if valid is None else valid[src_k]
    cq = int(np.prod(case.chunk_q))
    ck = int(np.prod(case.chunk_k))
    return dict(case=case, fx=fx, S=S, src_q=src_q, inv_q=inv_q, src_k=src_k, inv_k=inv_k,
                q=q, k=k, v=v, do=do, valid=valid, valid_re=valid_re, cq=cq, ck=ck)


def _tie_free_chunks(r):
    """q chunks with at least one row valid under the key-order mask."""
    nq = r["S"] // r["cq"]
    if r["valid_re"] is None:
        return np.ones(nq, bool)
    return r["valid_re"].reshape(nq, r["cq"]).any(axis=1)


@pytest.mark.parametrize("name", list(UNIFORM_CASES))
def test_uniform_layout_matches_reference(name):
    r = _setup(name)
    assert (r["src_q"] == r["fx"]["src_idx_q"]).all()
    assert (r["src_k"] == r["fx"]["src_idx_k"]).all()
    # inverse and padding rows
    assert (r["inv_q"][r["src_q"]] == np.arange(r["S"])).all()
    src, _ = O.uniform_layout(r["case"].grid_padded, r["case"].chunk_q, r["S"] + 64)
    assert (src[r["S"]:] == r["S"]).all()


def _select(r):
    case = r["case"]
    # q is pooled under the key-order mask, as the reference does for q and k of
    # one sequence (bsa_interface.py:609-610)
    return O.block_select_uniform(r["q"][:, r["src_q"]], r["k"][:, r["src_k"]], r["S"], r["S"],
                                  r["cq"], r["ck"], r["valid_re"], r["valid_re"], case.sparsity,
                                  case.cdf_threshold, want_chunks=True)


@pytest.mark.parametrize("name", list(UNIFORM_CASES))
def test_uniform_selection_matches_reference(name):
    r = _setup(name)
    bits_q, bits_k, sel = _select(r)
    nk = r["S"] // r["ck"]
    # unpadded grids: the reference pools and scores in bf16; the oracle (and the
    # CUDA path) in fp32, as the reference does whenever a valid mask exists
    key = "sel_chunks" if r["valid"] is not None else "sel_chunks_f32"
    ref = O.bits_to_dense(r["fx"][key], nk)
    ok = _tie_free_chunks(r)
    mine = sel.astype(bool)
    assert (mine[:, ok] == ref[:, ok]).all(), f"{(mine[:, ok] != ref[:, ok]).sum()} chunk pairs differ"
    # tile bitmaps: chunk selection expanded, tiles without a valid key dropped
    n_tiles = r["S"] // 64
    dense = O.bits_to_dense(bits_q, n_tiles)
    tq, tk = r["cq"] // 64, r["ck"] // 64
    exp = np.repeat(np.repeat(mine, tq, axis=1), tk, axis=2)
    if r["valid_re"] is not None:
        exp &= r["valid_re"].reshape(n_tiles, 64).any(axis=1)[None, None, :]
    assert (dense == exp).all()
    assert (O.bits_to_dense(bits_k, n_tiles) == dense.transpose(0, 2, 1)).all()


def _bits_from_chunks(sel, r):
    """Chunk-level selection [h, nq, nk] -> tile bitmap (tiles without a valid key dropped)."""
    n_tiles = r["S"] // 64
    tq, tk = r["cq"] // 64, r["ck"] // 64
    exp = np.repeat(np.repeat(sel.astype(bool), tq, axis=1), tk, axis=2)
    if r["valid_re"] is not None:
        exp &= r["valid_re"].reshape(n_tiles, 64).any(axis=1)[None, None, :]
    return O.dense_to_bits(exp)


@pytest.mark.parametrize("name", list(UNIFORM_CASES))
def test_uniform_attention_restatement(name):
    """The float64 restatement on the selection the reference's fp32 pass made
    (tie rows included, so dK / dV see every query row)."""
    r = _setup(name)
    nk = r["S"] // r["ck"]
    bits_q = _bits_from_chunks(O.bits_to_dense(r["fx"]["sel_chunks_f32"], nk), r)
    f = O.bf16_bits_to_f32
    qr, kr, vr = f(r["q"][:, r["src_q"]]), f(r["k"][:, r["src_k"]]), f(r["v"][:, r["src_k"]])
    o, lse = O.bsa_forward(qr, kr, vr, bits_q, r["valid_re"])
    dq, dk, dv = O.bsa_backward(qr, kr, vr, o, f(r["do"])[:, r["src_q"]], bits_q, r["valid_re"])
    fx, rows = r["fx"], r["fx"]["rows"]
    for nm, x, inv in (("o", o, r["inv_q"]), ("dq", dq, r["inv_q"]), ("dk", dk, r["inv_k"]),
                       ("dv", dv, r["inv_k"])):
        got = x[:, inv][:, rows]
        ref = fx[nm]
        err = np.abs(got - ref).max()
        assert err <= 1e-5 * max(1.0, np.abs(ref).max()), (nm, err)
