"""GPU parity of the selection side, through the C ABI, against the CPU oracle.

Everything here is integer / index work or floating-point work done in a fixed
order, so the bar is bit-exact equality (shape ids, permutation, tile maps,
zone statistics, selected tile pairs)."""
import numpy as np
import pytest
import torch

from helpers import bits, load_fixture
from inputs import CASES, Case, make_inputs
from oracle import oracle as O
from prism_b200 import ops

pytestmark = pytest.mark.gpu

EXTRA = {
    # reduced 720p-like grid with many zones and both block sizes, D = 128
    "grid_720p_slice": Case("grid_720p_slice", (21, 45, 24), 2, 128, values="zoned",
                            amp=(0.05, 1.0), sparsity=0.92, cdf_threshold=0.9, tau_128=0.35,
                            seed=70),
    # 40 heads exercise the head-average loop; penalty method
    "heads40": Case("heads40", (5, 13, 9), 40, 64, values="zoned", amp=(0.1, 1.0),
                    method="penalty", sparsity=0.8, cdf_threshold=0.7, tau_128=0.5, seed=80),
    # exact grid (no padding, valid mask None)
    "nopad_topk": Case("nopad_topk", (8, 16, 8), 2, 64, values="zoned", amp=(0.1, 1.0),
                       sparsity=0.7, cdf_threshold=None, seed=90),
}
ALL = dict(CASES, **EXTRA)


def _case_data(name, dev):
    case = ALL[name]
    inp = make_inputs(case)
    d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in inp.items()}
    return case, inp, d


@pytest.mark.parametrize("name", list(ALL))
def test_selection_pipeline_bit_exact(name, cuda):
    case, inp, d = _case_data(name, cuda)
    gp = case.grid_padded
    valid = d["valid"]
    norms = d["norms"]
    # zone statistics
    packed, av, audio = ops.zone_stats(d["v"][0], gp, gp, valid, norms)
    vb = bits(inp["v"][0])
    vm = None if inp["valid"] is None else inp["valid"].numpy().astype(np.uint8)
    nb_ = None if inp["norms"] is None else bits(inp["norms"])
    o_packed, o_av, o_audio = O.zone_stats(vb, gp, vm, nb_)
    assert np.array_equal(packed.cpu().numpy().view(np.uint32), o_packed.view(np.uint32))
    assert np.array_equal(av.cpu().numpy(), o_av)
    assert np.array_equal(audio.cpu().numpy().view(np.uint32), o_audio.view(np.uint32))
    # shape ids (+ g, rho diagnostics)
    ids, g, rho = ops.shape_select(packed, av, audio, norms is not None, case.method, case.lambda_a,
                                   case.tau_128, case.lambda_128, want_diag=True)
    o_ids, o_g, o_rho = O.shape_select(o_packed, o_av, o_audio, nb_ is not None, case.method,
                                       case.lambda_a, case.tau_128, case.lambda_128)
    assert np.array_equal(ids.cpu().numpy(), o_ids)
    assert np.array_equal(g.cpu().numpy().view(np.uint32), o_g.view(np.uint32))
    assert np.array_equal(rho.cpu().numpy().view(np.uint32), o_rho.view(np.uint32))
    if name in CASES:
        assert np.array_equal(o_ids, load_fixture(name)["shape_ids"])
    # layout
    lay = ops.build_layout(ids, gp)
    src, inv, bot, bt, nbk = O.layout(o_ids, gp)
    assert np.array_equal(lay["src_idx"].cpu().numpy(), src)
    assert np.array_equal(lay["inv_idx"].cpu().numpy(), inv)
    assert np.array_equal(lay["block_of_tile"].cpu().numpy(), bot)
    assert int(lay["n_blocks"].item()) == nbk
    assert np.array_equal(lay["block_tiles"].cpu().numpy()[: nbk + 1], bt)
    # key validity per tile
    tb, tc = ops.tile_valid(lay["src_idx"], valid, gp, gp)
    vre = np.ones(src.size, np.uint8) if vm is None else vm[src]
    exp_bits = np.packbits(vre.reshape(-1, 64).astype(bool), axis=1, bitorder="little").view(np.uint64)[:, 0]
    assert np.array_equal(tb.cpu().numpy().view(np.uint64), exp_bits)
    assert np.array_equal(tc.cpu().numpy(), vre.reshape(-1, 64).sum(1))
    # gather
    q_re = ops.gather_rows(d["q"][0], gp, gp, lay["src_idx"])
    k_re = ops.gather_rows(d["k"][0], gp, gp, lay["src_idx"])
    assert np.array_equal(bits(q_re), bits(inp["q"][0])[:, src])
    # pooled scores + hybrid selection
    bq, bk = ops.block_select(q_re, k_re, lay, tb, case.sparsity, case.cdf_threshold)
    o_bq, o_bk, _ = O.block_select(bits(q_re), bits(k_re), None if vm is None else vm[src], bt, nbk,
                                   case.sparsity, case.cdf_threshold)
    assert np.array_equal(bq.cpu().numpy().view(np.uint32), o_bq)
    assert np.array_equal(bk.cpu().numpy().view(np.uint32), o_bk)
    if name in CASES and valid is not None:
        nt = src.size // 64
        ref = O.bits_to_dense(load_fixture(name)["sel_bits"], nt)
        # rows of padding-only query blocks tie on every score; the reference's
        # choice there is torch.topk's unspecified tie order (see test_oracle_golden)
        tile_cnt = vre.reshape(-1, 64).sum(1)
        blk_cnt = np.array([sum(tile_cnt[j] for j in bt[b] if j < nt) for b in range(nbk)])
        real = blk_cnt[bot] > 0
        assert np.array_equal(O.bits_to_dense(o_bq, nt)[:, real], ref[:, real])
    # determinism: a second run is bit-identical
    bq2, _ = ops.block_select(q_re, k_re, lay, tb, case.sparsity, case.cdf_threshold)
    assert torch.equal(bq, bq2)


@pytest.mark.parametrize("name", [n for n in ALL if ALL[n].audio])
def test_token_norms_bit_exact(name, cuda):
    case, inp, d = _case_data(name, cuda)
    got = bits(ops.token_norms(d["a2v"]))
    assert np.array_equal(got, O.token_norms(bits(inp["a2v"])))
    if name in CASES:
        assert np.array_equal(got, load_fixture(name)["norms_u"])


def test_token_norms_wide(cuda):
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(777, 5120, generator=g) * 3).to(torch.bfloat16)
    assert np.array_equal(bits(ops.token_norms(x.to(cuda))), O.token_norms(bits(x)))


@pytest.mark.parametrize("name", ["mixed_d64", "grid_720p_slice", "heads40"])
def test_unpadded_source_grid_matches_padded(name, cuda):
    """Zone statistics / tile validity on the UNPADDED tensors (fused padding)
    equal those on the zero-padded tensors with the valid mask."""
    case, inp, d = _case_data(name, cuda)
    gp = case.grid_padded
    a = ops.zone_stats(d["v"][0], gp, gp, d["valid"], d["norms"])
    nu = None if d["norms_u"] is None else d["norms_u"]
    b = ops.zone_stats(d["v_u"][0], case.grid, gp, None, nu)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    # [S, H, D] strided layout reads the same values
    v_shd = d["v_u"][0].transpose(0, 1).contiguous()
    c = ops.zone_stats(v_shd.transpose(0, 1), case.grid, gp, None, nu)
    for x, y in zip(a, c):
        assert torch.equal(x, y)
    ids = ops.shape_select(*a, d["norms"] is not None, case.method)
    lay = ops.build_layout(ids, gp)
    t1 = ops.tile_valid(lay["src_idx"], d["valid"], gp, gp)
    t2 = ops.tile_valid(lay["src_idx"], None, case.grid, gp)
    assert torch.equal(t1[0], t2[0]) and torch.equal(t1[1], t2[1])
    g1 = ops.gather_rows(d["q"][0], gp, gp, lay["src_idx"])
    g2 = ops.gather_rows(d["q_u"][0], case.grid, gp, lay["src_idx"])
    assert torch.equal(g1, g2)


def test_invalid_arguments_raise(cuda):
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        ops.selection_mode(None, None)
    with pytest.raises(ValueError):
        ops.shape_select(torch.zeros(1, 25 * 64, device=cuda), torch.zeros(1, 24, dtype=torch.uint8, device=cuda),
                         torch.zeros(1, 25, device=cuda), False, "bogus")
    with pytest.raises(Exception):
        ops.token_norms(x[:, :7])


@pytest.mark.parametrize("D", [8, 16, 32, 256])
def test_zone_stats_head_dims_bit_exact(D, cuda):
    """Zone statistics and shape ids at head dims on both sides of the row-parallel
    kernel's range (16 <= D <= 128; the one-thread-per-channel-pair kernel otherwise),
    with 5 heads, padding on every axis and audio norms, against the C oracle."""
    g = torch.Generator().manual_seed(D)
    grid, gp, heads = (5, 11, 13), (8, 16, 16), 5
    S = grid[0] * grid[1] * grid[2]
    Sp = gp[0] * gp[1] * gp[2]
    v_pad = torch.zeros(heads, gp[0], gp[1], gp[2], D)
    v_pad[:, :grid[0], :grid[1], :grid[2]] = torch.randn(heads, *grid, D, generator=g)
    v_pad = v_pad.reshape(heads, Sp, D).to(torch.bfloat16)
    valid = torch.zeros(gp, dtype=torch.bool)
    valid[:grid[0], :grid[1], :grid[2]] = True
    valid = valid.reshape(Sp)
    norms = (torch.rand(Sp, generator=g) * 3).to(torch.bfloat16) * valid
    packed, av, audio = ops.zone_stats(v_pad.to(cuda), gp, gp, valid.to(cuda), norms.to(cuda))
    o_packed, o_av, o_audio = O.zone_stats(bits(v_pad), gp, valid.numpy().astype(np.uint8),
                                           bits(norms))
    assert np.array_equal(packed.cpu().numpy().view(np.uint32), o_packed.view(np.uint32))
    assert np.array_equal(av.cpu().numpy(), o_av)
    assert np.array_equal(audio.cpu().numpy().view(np.uint32), o_audio.view(np.uint32))
    ids = ops.shape_select(packed, av, audio, True, "ivpq")
    o_ids, _, _ = O.shape_select(o_packed, o_av, o_audio, True, "ivpq", 0.5, 0.15, 1.0)
    assert np.array_equal(ids.cpu().numpy(), o_ids)
    assert S < Sp
