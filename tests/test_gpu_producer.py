"""GPU parity of the producer / consumer fusion (prism_b200.producer): RMSNorm +
3D RoPE + all-to-all pack of q / k / v in one pass (wan_video_dit.py:699-705,
764-787), its backward, and the whole SelfAttention layer with the output
projection reading the inverse all-to-all's receive buffer (:824-841).

* forward: the kernel's bf16 q equals the oracle (torch.nn.RMSNorm restated, then
  the reference's rope_apply_head_dim restated bit for bit) and the reference's own
  outputs on nearly every element, within one rounding step elsewhere;
* packed layout: head padding, ranks, and an uneven last rank's zero rows;
* backward: against float64 torch autograd of the same math (rel-L2 1e-2);
* the fused layer equals the unfused composition at P = 1 (outputs and gradients)
  and, with the all-to-all emulated by buffer swaps on one GPU, at P = 2.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import bits, load_fixture, rel_l2
from inputs import PRODUCER_CASES, make_producer_inputs
from oracle import oracle as O
from prism_b200 import ops, run_bsa_uniform
from prism_b200.linear import linear
from prism_b200.producer import (fused_self_attention, norm_rope_pack, o_proj_packed, rope_table,
                                 rope_table_ff)

pytestmark = pytest.mark.gpu


def _ulps(a_bits, b_bits):
    """bf16 values as float32 -> |a - b| in units of b's last place (>= 2^-133)."""
    a = O.bf16_bits_to_f32(a_bits).astype(np.float64)
    b = O.bf16_bits_to_f32(b_bits).astype(np.float64)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(b), 2.0 ** -126))) - 7)
    return np.abs(a - b) / ulp


@pytest.mark.parametrize("name", list(PRODUCER_CASES))
def test_norm_rope_forward(name, cuda):
    grid, heads, D, seed = PRODUCER_CASES[name]
    fx = load_fixture(name)
    x, gamma = make_producer_inputs(grid, heads, D, seed)
    S = x.shape[1]
    cs = rope_table_ff(rope_table(grid, D, device=cuda))
    q_pk, rstd = ops.norm_rope_pack(x[0].to(cuda), heads, 1, heads, S, gamma.to(cuda).float(), 1e-6, cs,
                                    True)
    got = bits(q_pk.view(S, heads * D))
    ref = O.rope_apply(O.rms_norm(bits(x[0]), gamma.float().numpy()), fx["freqs"], D)
    for r, what in ((ref, "oracle"), (fx["y"], "reference")):
        u = _ulps(got, r)
        assert (u == 0).mean() >= 0.98 and u.max() <= 4, (what, (u == 0).mean(), u.max())
    # rstd = 1 / sqrt(mean(x^2) + eps)
    xf = x[0].double()
    ref_r = 1.0 / torch.sqrt((xf ** 2).mean(-1) + 1e-6)
    assert torch.allclose(rstd.cpu().double(), ref_r, rtol=1e-5)


def test_pack_layout(cuda):
    """P ranks x hp heads with padding heads and a padded last shard."""
    grid, heads, D, seed = (2, 3, 5), 3, 128, 7
    x, gamma = make_producer_inputs(grid, heads, D, seed)
    S = x.shape[1]
    cs = rope_table_ff(rope_table(grid, D, device=cuda))
    xc, gc = x[0].to(cuda), gamma.to(cuda).float()
    ref, _ = ops.norm_rope_pack(xc, heads, 1, heads, S, gc, 1e-6, cs, True)
    ref = ref.view(S, heads, D)
    for P, norm in ((2, True), (4, True), (2, False)):
        hp = -(-heads // P)
        S_pack = S + 3
        pk, _ = ops.norm_rope_pack(xc, heads, P, hp, S_pack, gc, 1e-6, cs, norm)
        want = ref if norm else xc.view(S, heads, D)
        for p in range(P):
            for hh in range(hp):
                h = p * hp + hh
                blk = pk[p, :S, hh]
                if h < heads:
                    assert torch.equal(blk, want[:, h])
                else:
                    assert not blk.any()
            assert not pk[p, S:].any()


@pytest.mark.parametrize("name", list(PRODUCER_CASES))
def test_norm_rope_backward(name, cuda):
    grid, heads, D, seed = PRODUCER_CASES[name]
    x, gamma = make_producer_inputs(grid, heads, D, seed)
    S, C = x.shape[1], heads * D
    cs = rope_table(grid, D, device=cuda)
    ff = rope_table_ff(cs)
    gen = torch.Generator().manual_seed(seed + 50)
    g = torch.randn(S, C, generator=gen).to(torch.bfloat16)
    xc, gc = x[0].to(cuda), gamma.to(cuda).float()
    _, rstd = ops.norm_rope_pack(xc, heads, 1, heads, S, gc, 1e-6, ff, True)
    dx, dgamma = ops.norm_rope_pack_bwd(g.to(cuda).view(1, S, heads, D), xc, heads, S, gc, rstd, ff, True)
    # float64 reference of the same math
    x64 = x[0].double().requires_grad_(True)
    g64 = gamma.double().requires_grad_(True)
    y = x64 * torch.rsqrt((x64 ** 2).mean(-1, keepdim=True) + 1e-6) * g64
    yc = torch.view_as_complex(y.view(S, heads, D // 2, 2).contiguous())
    f = torch.view_as_complex(cs.cpu().view(S, 1, D // 2, 2).contiguous())
    out = torch.view_as_real(yc * f).reshape(S, C)
    (out * g.double()).sum().backward()
    assert rel_l2(dx.float().cpu().numpy(), x64.grad.numpy()) <= 1e-2
    assert rel_l2(dgamma.cpu().numpy(), g64.grad.numpy()) <= 1e-2
    # v: the unpack alone
    dv, _ = ops.norm_rope_pack_bwd(g.to(cuda).view(1, S, heads, D), None, heads, S, norm=False)
    assert torch.equal(dv.cpu(), g)


def _params(dim, gen, device):
    mk = lambda *s: (torch.randn(*s, generator=gen) / s[-1] ** 0.5).to(torch.bfloat16).to(device)
    p = {n: mk(dim, dim) for n in ("q_weight", "k_weight", "v_weight", "o_weight")}
    p.update({n: (0.1 * torch.randn(dim, generator=gen)).to(torch.bfloat16).to(device)
              for n in ("q_bias", "k_bias", "v_bias", "o_bias")})
    p["norm_q_weight"] = (1 + 0.1 * torch.randn(dim, generator=gen)).to(device)
    p["norm_k_weight"] = (1 + 0.1 * torch.randn(dim, generator=gen)).to(device)
    p["eps"] = 1e-6
    return p


ATTN = dict(sparsity=0.5, cdf_threshold=None, chunk_3d_shape_q=(4, 4, 4), chunk_3d_shape_k=(4, 4, 4))


def test_fused_layer_equals_unfused_p1(cuda):
    grid, heads, D = (4, 8, 12), 4, 128
    dim = heads * D
    gen = torch.Generator().manual_seed(11)
    S = grid[0] * grid[1] * grid[2]
    x = (torch.randn(1, S, dim, generator=gen)).to(torch.bfloat16).to(cuda)
    params = _params(dim, gen, cuda)
    for p in params.values():
        if torch.is_tensor(p):
            p.requires_grad_(True)
    cs = rope_table(grid, D, device=cuda)
    xa = x.clone().requires_grad_(True)
    out = fused_self_attention(xa, cs, params, heads, grid, attention="uniform", **ATTN)
    gout = torch.randn(out.shape, generator=gen).to(torch.bfloat16).to(cuda)
    out.backward(gout)
    ga = {n: p.grad.clone() for n, p in params.items() if torch.is_tensor(p)}
    gx = xa.grad.clone()
    for p in params.values():
        if torch.is_tensor(p):
            p.grad = None
    # unfused composition with the same kernels: projections, norm_rope_pack at P = 1,
    # attention, output projection as one GEMM
    def unfused(proj):
        xb = x.clone().requires_grad_(True)
        ql, kl, vl = (proj(xb[0], params[n + "_weight"], params[n + "_bias"]) for n in "qkv")
        q, k, v = norm_rope_pack(ql, kl, vl, params["norm_q_weight"], params["norm_k_weight"], 1e-6,
                                 cs, heads)
        xo = run_bsa_uniform(q.view(1, S, heads, D), k.view(1, S, heads, D), v.view(1, S, heads, D),
                             grid, layout="bshd", **ATTN)
        ref = proj(xo.reshape(S, dim), params["o_weight"], params["o_bias"]).unsqueeze(0)
        ref.backward(gout)
        grads = {n: p.grad.clone() for n, p in params.items() if torch.is_tensor(p)}
        for p in params.values():
            if torch.is_tensor(p):
                p.grad = None
        return ref, xb.grad, grads

    ref, gxb, gb = unfused(linear)
    assert torch.equal(out, ref)
    assert torch.equal(gx, gxb)
    for n in ga:
        assert torch.equal(ga[n], gb[n]), n
    # the repository's GEMM against cuBLAS (F.linear) through the whole layer: bf16 rounding
    ref2, gx2, g2 = unfused(F.linear)
    for name, a, b in [("out", out, ref2), ("dx", gx, gx2)] + [(n, ga[n], g2[n]) for n in ga]:
        a, b = a.float(), b.float()
        assert float((a - b).norm() / b.norm()) <= 1e-2, name


def test_fused_layer_two_rank_emulation(cuda):
    """Ulysses at P = 2 on one GPU: each rank's pack, the all-to-all as buffer swaps,
    the attention on each rank's heads, the inverse exchange and the K-split output
    projection, against the P = 1 layer (uneven split: 196 tokens over 2 ranks is
    even; 3 x 7 x 9 = 189 is not)."""
    for grid in ((4, 7, 7), (3, 7, 9)):
        heads, D = 4, 128
        dim = heads * D
        gen = torch.Generator().manual_seed(21)
        S = grid[0] * grid[1] * grid[2]
        x = torch.randn(1, S, dim, generator=gen).to(torch.bfloat16).to(cuda)
        params = _params(dim, gen, cuda)
        cs = rope_table(grid, D, device=cuda)
        with torch.no_grad():
            ref = fused_self_attention(x, cs, params, heads, grid, attention="uniform", **ATTN)
            P, hp = 2, heads // 2
            S_pack = -(-S // P)
            sizes = [S_pack, S - S_pack]
            rows = [slice(0, sizes[0]), slice(sizes[0], S)]
            send = []
            for r in range(P):
                xr = x[0, rows[r]]
                ql, kl, vl = (linear(xr, params[n + "_weight"], params[n + "_bias"]) for n in "qkv")
                send.append(norm_rope_pack(ql, kl, vl, params["norm_q_weight"], params["norm_k_weight"],
                                           1e-6, cs[rows[r]].contiguous(), heads, P, hp, S_pack))
            recv = [[torch.stack([send[p][t][r] for p in range(P)]) for t in range(3)] for r in range(P)]
            xo = []
            for r in range(P):
                q4, k4, v4 = (t.view(1, P * S_pack, hp, D)[:, :S] for t in recv[r])
                o = run_bsa_uniform(q4, k4, v4, grid, layout="bshd", **ATTN)
                xo.append(F.pad(o, (0, 0, 0, 0, 0, P * S_pack - S)).reshape(P, S_pack, hp, D))
            outs = []
            for r in range(P):
                back = torch.stack([xo[p][r] for p in range(P)])
                outs.append(o_proj_packed(back, params["o_weight"], params["o_bias"], heads, sizes[r]))
            got = torch.cat(outs, 0).unsqueeze(0)
        assert rel_l2(got.float().cpu().numpy(), ref.float().cpu().numpy()) <= 5e-3
        assert (got.float() - ref.float()).abs().max().item() <= 2e-2
