"""Producer / consumer fusion around the attention core: the whole
``SelfAttention.forward`` of the video DiT (hymm/models/modules/wan_video_dit.py:
689-841) with the attention in between.

Reference sequence (per layer, per rank):
  q = norm_q(self.q(x)); k = norm_k(self.k(x)); v = self.v(x)          (:699-701)
  q, k = rope_apply_head_dim(q / k, freqs)  (float64 complex)           (:704-705)
  q, k, v -> [B, S/P, H, D] -> head padding -> all_to_all_4D             (:764-787)
  attention on the local heads                                          (:795-823)
  all_to_all_4D back -> drop padded heads -> flatten -> self.o(x)         (:824-841)

Here:
* the projections run on the repository's tensor-core GEMM (prism_b200.linear,
  prism_gemm_bf16), forward and backward;
* RMSNorm + RoPE + the all-to-all pack are one pass per token row
  (``prism_norm_rope_pack``), writing each head straight into the send layout
  [P, S/P, H/P, D], and the backward is the mirror pass (``prism_norm_rope_pack_bwd``):
  the reference moves q and k through HBM five to six times between the GEMM and
  the all-to-all (norm in fp32, bf16 copy, fp64 copy, rotated fp64, bf16 copy,
  packed copy);
* the all-to-all exchanges those buffers as they are (NCCL all_to_all_single) and
  the attention reads the received buffer in place;
* the output projection reads the inverse all-to-all's receive buffer in place:
  out = sum over source ranks p of recv[p] W_o[:, heads of p]^T, P accumulating
  GEMMs instead of an unpack copy plus one GEMM (prism_b200.linear.o_proj_packed).

``rope_table`` restates ``precompute_freqs_cis_3d`` (:125-139) and the per-token
assembly of :1183-1187 as a (cos, sin) float64 table; the kernels take it split into
float hi + lo parts (``rope_table_ff``) and evaluate the rotation in float-float
arithmetic, which reproduces the reference's float64 evaluation after its rounding
to bf16.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import ops
from .linear import linear, o_proj_packed
from .communications import (HeadsToWire, WireToHeads, live_ranks, sp_chunk_sizes,
                             sp_num_local_real_heads, sp_pad_num_heads)
from .parallel_states import get_sequence_parallel_state, nccl_info


def _freqs_1d(dim: int, end: int, theta: float) -> torch.Tensor:
    """precompute_freqs_cis (wan_video_dit.py:133-139): complex128 [end, dim/2]."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].double() / dim))
    ang = torch.outer(torch.arange(end), inv)
    return torch.polar(torch.ones_like(ang), ang)


def rope_table(grid: Tuple[int, int, int], head_dim: int, theta: float = 10000.0, end: int = 1024,
               device=None) -> torch.Tensor:
    """(cos, sin) of the 3D RoPE of every token of grid (T, H, W), THW order:
    float64 [T*H*W, head_dim/2, 2].  Frame / height / width frequencies take
    head_dim - 2*(head_dim//3), head_dim//3, head_dim//3 dimensions
    (precompute_freqs_cis_3d, wan_video_dit.py:125-130; assembly :1183-1187)."""
    f, h, w = (int(g) for g in grid)
    d_hw = head_dim // 3
    ff = _freqs_1d(head_dim - 2 * d_hw, end, theta)
    fh = _freqs_1d(d_hw, end, theta)
    fw = _freqs_1d(d_hw, end, theta)
    freqs = torch.cat([ff[:f].view(f, 1, 1, -1).expand(f, h, w, -1),
                       fh[:h].view(1, h, 1, -1).expand(f, h, w, -1),
                       fw[:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(f * h * w, -1)
    if freqs.shape[1] != head_dim // 2:
        raise ValueError(f"the 3D RoPE split of head_dim {head_dim} gives {freqs.shape[1]} frequency "
                         f"pairs, not {head_dim // 2} (the reference's rope_apply_head_dim fails too)")
    return torch.view_as_real(freqs).contiguous().to(device)


def rope_table_ff(table: torch.Tensor) -> torch.Tensor:
    """A float64 (cos, sin) table [S, D/2, 2] -> the kernels' float-float form
    [S, D/2, 4] fp32 = (cos_hi, cos_lo, sin_hi, sin_lo), hi = float(x),
    lo = float(x - hi)."""
    if table.dtype == torch.float32 and table.shape[-1] == 4:
        return table
    hi = table.to(torch.float32)
    lo = (table - hi.to(torch.float64)).to(torch.float32)
    return torch.stack([hi[..., 0], lo[..., 0], hi[..., 1], lo[..., 1]], dim=-1).contiguous()


class _NormRopePack(torch.autograd.Function):
    """(q_lin, k_lin, v_lin) [S, H*D] -> packed (q, k, v) [P, S_pack, hp, D]."""

    @staticmethod
    def forward(ctx, q_lin, k_lin, v_lin, gamma_q, gamma_k, eps, rope_cs, heads, P, hp, S_pack):
        q_pk, rq = ops.norm_rope_pack(q_lin, heads, P, hp, S_pack, gamma_q, eps, rope_cs, True)
        k_pk, rk = ops.norm_rope_pack(k_lin, heads, P, hp, S_pack, gamma_k, eps, rope_cs, True)
        v_pk, _ = ops.norm_rope_pack(v_lin, heads, P, hp, S_pack, norm=False)
        ctx.save_for_backward(q_lin, k_lin, gamma_q, gamma_k, rq, rk, rope_cs)
        ctx.meta = (heads, q_lin.shape[0])
        return q_pk, k_pk, v_pk

    @staticmethod
    def backward(ctx, gq, gk, gv):
        q_lin, k_lin, gamma_q, gamma_k, rq, rk, cs = ctx.saved_tensors
        heads, S = ctx.meta
        z = lambda g, ref: torch.zeros_like(ref) if g is None else g
        ref = gq if gq is not None else (gk if gk is not None else gv)
        dq, dgq = ops.norm_rope_pack_bwd(z(gq, ref), q_lin, heads, S, gamma_q, rq, cs, True)
        dk, dgk = ops.norm_rope_pack_bwd(z(gk, ref), k_lin, heads, S, gamma_k, rk, cs, True)
        dv, _ = ops.norm_rope_pack_bwd(z(gv, ref), None, heads, S, norm=False)
        dgq = None if gamma_q is None else dgq.to(gamma_q.dtype)
        dgk = None if gamma_k is None else dgk.to(gamma_k.dtype)
        return dq, dk, dv, dgq, dgk, None, None, None, None, None, None


def norm_rope_pack(q_lin, k_lin, v_lin, gamma_q, gamma_k, eps: float, rope_cs, heads: int,
                   P: int = 1, hp: Optional[int] = None, S_pack: Optional[int] = None):
    """RMSNorm + 3D RoPE of q / k and the all-to-all pack of q / k / v (differentiable).
    rope_cs: rope_table's float64 table or its rope_table_ff form."""
    rope_cs = rope_table_ff(rope_cs)
    hp = heads if hp is None else hp
    S_pack = q_lin.shape[0] if S_pack is None else S_pack
    return _NormRopePack.apply(q_lin, k_lin, v_lin, gamma_q, gamma_k, float(eps), rope_cs, heads, P,
                               hp, S_pack)


def fused_self_attention(x: torch.Tensor, rope_cs: torch.Tensor, params: dict, num_heads: int,
                         grid_size: Tuple[int, int, int], *, attention: str = "dynamic",
                         full_seq_len: Optional[int] = None,
                         a2v_bridge_residual: Optional[torch.Tensor] = None, **attn_kw):
    """SelfAttention.forward (wan_video_dit.py:689-841) with the fused producer /
    consumer.  x [1, S_local, dim] (this rank's tokens, THW order); rope_cs
    [S_local, D/2, 2] float64 (this rank's rows of rope_table); params: q_weight,
    q_bias, k_weight, k_bias, v_weight, v_bias, o_weight, o_bias [dim(, dim)],
    norm_q_weight, norm_k_weight [dim], eps.  attention: "dynamic" (run_bsa_dynamic,
    kwargs method, sparsity, cdf_threshold, lambda_a, tau_128, lambda_128) or
    "uniform" (run_bsa_uniform, kwargs sparsity, cdf_threshold, chunk_3d_shape_q/k).
    Returns [1, S_local, dim]."""
    from .attention import audio_token_norms
    from .bsa_interface import run_bsa_uniform
    from .dynamic_block_attention import run_bsa_dynamic

    b, S_local, dim = x.shape
    assert b == 1, "batch 1"
    D = dim // num_heads
    xs = x[0]
    q_lin = linear(xs, params["q_weight"], params.get("q_bias"))
    k_lin = linear(xs, params["k_weight"], params.get("k_bias"))
    v_lin = linear(xs, params["v_weight"], params.get("v_bias"))
    sp = get_sequence_parallel_state() and nccl_info.sp_size > 1
    P = nccl_info.sp_size if sp else 1
    padded = sp_pad_num_heads(num_heads, P)
    hp = padded // P
    S_full = int(full_seq_len) if (sp and full_seq_len is not None) else S_local * P
    S_pack = sp_chunk_sizes(S_full, P)[0] if sp else S_local
    q_pk, k_pk, v_pk = norm_rope_pack(q_lin, k_lin, v_lin, params.get("norm_q_weight"),
                                      params.get("norm_k_weight"), params.get("eps", 1e-6), rope_cs,
                                      num_heads, P, hp, S_pack)
    if sp:
        # exchange; the full sequence of this rank's hp heads as [1, S_full, hp, D]
        # views of the receive buffers
        group = nccl_info.sp_group
        q4, k4, v4 = (WireToHeads.apply(t.unsqueeze(1), group, S_full) for t in (q_pk, k_pk, v_pk))
    else:
        q4, k4, v4 = (t.view(1, S_local, hp, D) for t in (q_pk, k_pk, v_pk))
    rank = nccl_info.rank_within_spgroup if sp else 0
    local = sp_num_local_real_heads(num_heads, padded, P, rank)
    norms = audio_token_norms(a2v_bridge_residual, full_seq_len)
    if local > 0:
        q4, k4, v4 = (t[:, :, :local] for t in (q4, k4, v4))
        if attention == "dynamic":
            xo = run_bsa_dynamic(q4, k4, v4, grid_size, audio_token_norms=norms, layout="bshd",
                                 seq_capacity=P * S_pack if sp else None,
                                 sp_live_ranks=live_ranks(num_heads, P) if sp else None, **attn_kw)
        elif attention == "uniform":
            xo = run_bsa_uniform(q4, k4, v4, grid_size, layout="bshd", **attn_kw)
        else:
            raise ValueError(f"attention must be 'dynamic' or 'uniform', got {attention!r}")
        if local != hp:
            xo = F.pad(xo, (0, 0, 0, hp - local))
    else:
        # padding-only rank: stay connected to the graph so that the backward
        # all-to-alls fire on every rank (wan_video_dit.py:814-823); a dynamic
        # layer's zone statistics all-reduce is joined as the local attention would
        if attention == "dynamic" and attn_kw.get("shape_ids") is None:
            from .dynamic_block_shape import _maybe_sp_average
            Tp, Hp_, Wp = ops.padded_grid(grid_size)
            _maybe_sp_average(torch.zeros((Tp // 8) * (Hp_ // 8) * (Wp // 8), 25 * D, device=x.device),
                              live_ranks=live_ranks(num_heads, P))
        xo = (q4 + k4 + v4) * 0.0
    if sp:
        # sent as it is when xo is the attention's output buffer of P * S_pack rows
        recv = HeadsToWire.apply(xo, nccl_info.sp_group, S_full).squeeze(1)
    else:
        recv = xo.reshape(1, S_local, hp, D)
    out = o_proj_packed(recv, params["o_weight"], params.get("o_bias"), num_heads, S_local)
    return out.unsqueeze(0)


__all__ = ["rope_table", "rope_table_ff", "norm_rope_pack", "o_proj_packed", "fused_self_attention"]
