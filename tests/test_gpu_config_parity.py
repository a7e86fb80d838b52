"""Parity at the benchmark configurations' grids (2 and 3).

Config 1 (720p: 21x45x80 -> 24x48x80, 1,440 tiles) on 2 heads, config 2 (1080p:
21x68x120 -> 24x72x120, 3,240 tiles) on 1 head and config 3 (2K: 31x90x160 ->
32x96x160, 7,680 tiles) on 1 head, D = 128, zone-structured q/k/v, top-k 8 % (5 % for
config 3) + cumulative mass 0.9, audio token norms:

* selection side against the C oracle (oracle/prism_oracle.c) on the same inputs:
  shape ids, the permutation and both tile bitmaps bit for bit.  A differing
  selection would have to be a near-tie (score gap or |cdf - p| below 1e-6
  relative); the counts of differing zones / bitmap words are printed and must be 0;
* attention: EVERY real row of O, dQ, dK and dV against a float64 restatement of
  the block-sparse attention (helpers.torch_bsa_reference, run on the GPU because
  the grid is too large for the numpy oracle; tests/test_oracle_golden pins it to
  the numpy oracle), within max-abs 2e-2 and relative L2 1e-2 (north_star's bar).

Reference: bsa_interface.py:284-304 (selection), dynamic_block_attention.py:194-332
(the dynamic path), flash_attn_bsa_varlen_mask.py:193-1014 (kernels)."""
import math

import numpy as np
import pytest
import torch

from helpers import bits, torch_bsa_reference
from inputs import Case, make_inputs
from oracle import oracle as O
from prism_b200.dynamic_block_attention import run_bsa_dynamic

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-2, 1e-2

CONFIG_CASES = {
    "c1_720p_h2": Case("c1_720p_h2", (21, 45, 80), 2, 128, values="zoned", sparsity=0.92,
                       cdf_threshold=0.9, audio_tokens=64, seed=0),
    "c2_1080p_h1": Case("c2_1080p_h1", (21, 68, 120), 1, 128, values="zoned", sparsity=0.92,
                        cdf_threshold=0.9, audio_tokens=64, seed=1),
    # config 3's grid and selection rule (top-k 5 % + cumulative mass 0.9): 7,680 tiles,
    # ~50 M selected tile pairs on one head (the C oracle takes ~25 s on the host)
    "c3_2k_h1": Case("c3_2k_h1", (31, 90, 160), 1, 128, values="zoned", sparsity=0.95,
                     cdf_threshold=0.9, audio_tokens=64, seed=2),
}


def _to_tile_order(x_thw, grid, grid_padded, src):
    """[h, S, D] in unpadded THW order -> [h, S_p, D] tile order (padding rows zero)."""
    T, H, W = grid
    Tp, Hp, Wp = grid_padded
    h, S, D = x_thw.shape
    pad = torch.zeros(h, Tp, Hp, Wp, D, dtype=x_thw.dtype, device=x_thw.device)
    pad[:, :T, :H, :W] = x_thw.reshape(h, T, H, W, D)
    return pad.reshape(h, Tp * Hp * Wp, D)[:, src]


@pytest.mark.parametrize("name", list(CONFIG_CASES))
def test_config_grid_parity(name, cuda):
    case = CONFIG_CASES[name]
    inp = make_inputs(case)
    gp = case.grid_padded
    h, D = case.heads, case.head_dim
    qu, ku, vu = (inp[n + "_u"].to(cuda).requires_grad_(True) for n in ("q", "k", "v"))
    out, ids, plan = run_bsa_dynamic(qu, ku, vu, case.grid, method=case.method,
                                     sparsity=case.sparsity, cdf_threshold=case.cdf_threshold,
                                     audio_token_norms=inp["norms_u"].to(cuda),
                                     return_shape_ids=True, return_plan=True)
    out.backward(inp["do_u"].to(cuda))
    torch.cuda.synchronize()

    # ---- selection side against the C oracle
    valid = inp["valid"].numpy().astype(np.uint8)
    r = O.dynamic_forward_selection(bits(inp["q"][0]), bits(inp["k"][0]), bits(inp["v"][0]), gp,
                                    method=case.method, sparsity=case.sparsity,
                                    cdf_threshold=case.cdf_threshold,
                                    norms_bits=bits(inp["norms"]), valid=valid)
    ids_diff = int((ids.cpu().numpy() != r["shape_ids"]).sum())
    src_diff = int((plan.src_idx.cpu().numpy() != r["src_idx"]).sum())
    bq = plan.bits_q.cpu().numpy().view(np.uint32)
    bk = plan.bits_k.cpu().numpy().view(np.uint32)
    bq_diff = int((bq != r["bits_q"]).sum())
    bk_diff = int((bk != r["bits_k"]).sum())
    nt = bq.shape[1]
    pairs = int(np.unpackbits(bq.view(np.uint8)).sum())
    print(f"{name}: zones {ids.numel()}, differing shape ids {ids_diff}; permutation entries "
          f"differing {src_diff}; bitmap words differing q {bq_diff} / k {bk_diff}; selected "
          f"tile pairs {pairs} (density {pairs / (h * nt * nt):.3f})")
    assert ids_diff == 0 and src_diff == 0 and bq_diff == 0 and bk_diff == 0

    # ---- attention: every real row against the float64 restatement
    src = plan.src_idx
    q_re, k_re, v_re, do_re = (inp[n][0].to(cuda)[:, src] for n in ("q", "k", "v", "do"))
    o64, lse64, dq64, dk64, dv64 = torch_bsa_reference(q_re, k_re, v_re, do_re, plan.bits_q,
                                                       plan.tile_bits, 1.0 / math.sqrt(D))
    real = torch.from_numpy(valid).to(cuda).bool()[src]
    for label, got, ref in (("O", out.detach()[0], o64), ("dQ", qu.grad[0], dq64),
                            ("dK", ku.grad[0], dk64), ("dV", vu.grad[0], dv64)):
        g = _to_tile_order(got, case.grid, gp, src)[:, real].double()
        rf = ref[:, real]
        mx = float((g - rf).abs().max())
        rel = float((g - rf).norm() / max(float(rf.norm()), 1e-30))
        print(f"{name} {label}: max-abs {mx:.3e} rel-L2 {rel:.3e} over {int(real.sum()) * h} rows")
        assert math.isfinite(mx) and mx <= MAX_ABS and rel <= REL_L2, (label, mx, rel)
