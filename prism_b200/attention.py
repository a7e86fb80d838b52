"""Video self-attention core with Ulysses sequence parallelism.

``dynamic_self_attention`` is the part of ``SelfAttention.forward``
(hymm/models/modules/wan_video_dit.py:689-841) between the q/k/v projections
(+ RMSNorm + RoPE, done by the caller) and the output projection ``self.o``,
for the dynamic block-shape path:

* audio token norms from the a2v bridge residual, all-gathered over SP
  (:739-757);
* head padding + sequence->heads all-to-all of q, k, v (:764-787);
* dynamic block-sparse attention on the local heads (:795-812 ->
  ``_run_bsa_dynamic``), reading the all-to-all output in its [B, S, H, D]
  layout directly (the reference's permute().contiguous() copies are fused
  into the gather kernel);
* padding-only ranks stay connected to the graph (:814-823);
* heads->sequence all-to-all of the output and head truncation (:824-828).

``uniform_self_attention`` is the same branch for the uniform fixed-shape path
(the plain-BSA dispatch, :470-560).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops
from .communications import (HeadGeometry, ShardGeometry, all_gather, all_to_all_4D,
                             live_ranks, sp_pad_heads)
from .bsa_interface import run_bsa_uniform
from .dynamic_block_attention import run_bsa_dynamic
from .parallel_states import get_sequence_parallel_state, nccl_info


def audio_token_norms(a2v_bridge_residual: Optional[torch.Tensor], full_seq_len: Optional[int] = None):
    """||a2v[m]||_2 per token (bf16), all-gathered over SP (wan_video_dit.py:739-752)."""
    if a2v_bridge_residual is None:
        return None
    with torch.no_grad():
        local = ops.token_norms(a2v_bridge_residual)  # [B, S_local]
        if get_sequence_parallel_state():
            full = all_gather(local.unsqueeze(-1), dim=1, group=nccl_info.sp_group,
                              full_seq_len=full_seq_len)
            return full.squeeze(-1)[0]
        return local[0]


def _sp_self_attention(q, k, v, num_heads: int, full_seq_len, run_local, idle_local=None):
    """The Ulysses SP branch of SelfAttention.forward (wan_video_dit.py:764-828)
    around a local attention.  q, k, v: [B=1, S_local, num_heads*D].
    run_local(q4, k4, v4, ctx) gets [1, S, h, D] views (bshd) of the local heads'
    receive buffers and returns (x [1, S, h, D], extra); ctx carries
    ``seq_capacity`` (rows of the exchange buffers: an output stored in such a
    buffer is sent back without a copy) and ``live_ranks`` (ranks with real
    heads).  idle_local(ctx) runs on a rank that holds only padding heads, before
    its output exchange (collectives the local attention would have joined).
    Returns (x [B, S_local, num_heads*D], extra)."""
    b, s_local, hd = q.shape
    D = hd // num_heads
    q4, k4, v4 = (t.view(b, s_local, num_heads, D) for t in (q, k, v))
    if not get_sequence_parallel_state():
        x, extra = run_local(q4, k4, v4, {"seq_capacity": None, "live_ranks": None})
        return x.flatten(2), extra
    P = nccl_info.sp_size
    rank = nccl_info.rank_within_spgroup
    group = nccl_info.sp_group
    S = int(full_seq_len) if full_seq_len is not None else s_local * P
    heads = HeadGeometry(P, num_heads)
    padded = heads.hp * P
    if padded != num_heads:
        q4, k4, v4 = (sp_pad_heads(t, padded) for t in (q4, k4, v4))
    q4, k4, v4 = (all_to_all_4D(t, group, 2, 1, S) for t in (q4, k4, v4))
    hpr = heads.hp
    local = heads.real_on(rank)
    ctx = {"seq_capacity": P * ShardGeometry(P, S).C, "live_ranks": live_ranks(num_heads, P)}
    extra = None
    if local > 0:
        if local != hpr:
            q4, k4, v4 = q4[:, :, :local], k4[:, :, :local], v4[:, :, :local]
        x, extra = run_local(q4, k4, v4, ctx)
        if x.shape[2] != hpr:
            x = sp_pad_heads(x, hpr)
    else:
        # padding-only rank: keep the graph connected so the backward
        # exchanges fire symmetrically on every rank (wan_video_dit.py:814-823)
        if idle_local is not None:
            idle_local(ctx)
        x = (q4 + k4 + v4) * 0.0
    x = all_to_all_4D(x, group, 1, 2, S)
    if padded != num_heads:
        x = x[:, :, :num_heads]
    return x.flatten(2), extra


def dynamic_self_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           grid_size: Tuple[int, int, int], num_heads: int, *,
                           a2v_bridge_residual: Optional[torch.Tensor] = None,
                           full_seq_len: Optional[int] = None, method: str = "ivpq",
                           sparsity: Optional[float] = 0.9375,
                           cdf_threshold: Optional[float] = None, lambda_a: float = 0.5,
                           tau_128: float = 0.15, lambda_128: float = 1.0,
                           shape_ids: Optional[torch.Tensor] = None,
                           return_shape_ids: bool = False):
    """q, k, v: [B=1, S_local, num_heads*D] (projected, normed, rotated).
    Returns x [B, S_local, num_heads*D] (input of the output projection)."""
    D = q.shape[2] // num_heads
    norms = audio_token_norms(a2v_bridge_residual, full_seq_len)
    kw = dict(method=method, sparsity=sparsity, cdf_threshold=cdf_threshold, lambda_a=lambda_a,
              tau_128=tau_128, lambda_128=lambda_128, shape_ids=shape_ids, return_shape_ids=True,
              audio_token_norms=norms, layout="bshd")

    def idle(ctx):
        # the zone statistics all-reduce must still be joined (with zeros; the
        # average divides by the ranks that hold real heads)
        if shape_ids is None:
            from .dynamic_block_shape import _maybe_sp_average
            Tp, Hp, Wp = ops.padded_grid(grid_size)
            Nz = (Tp // 8) * (Hp // 8) * (Wp // 8)
            _maybe_sp_average(torch.zeros(Nz, 25 * D, device=q.device), live_ranks=ctx["live_ranks"])

    def local(a, b_, c, ctx):
        return run_bsa_dynamic(a, b_, c, grid_size, seq_capacity=ctx["seq_capacity"],
                               sp_live_ranks=ctx["live_ranks"], **kw)

    x, used = _sp_self_attention(q, k, v, num_heads, full_seq_len, local, idle)
    used = shape_ids if used is None else used
    if return_shape_ids:
        return x, used
    return x


def uniform_self_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           grid_size: Tuple[int, int, int], num_heads: int, *,
                           full_seq_len: Optional[int] = None,
                           sparsity: Optional[float] = 0.875,
                           cdf_threshold: Optional[float] = None,
                           chunk_3d_shape_q=(4, 4, 4), chunk_3d_shape_k=(4, 4, 4),
                           a2v_bridge_residual: Optional[torch.Tensor] = None,
                           audio_gate=None, audio_boost_gamma=None,
                           audio_weighted_lambda: float = 0.0,
                           variance_boost_gamma: float = 0.0,
                           correction: Optional[str] = None, taylor_alpha_f: float = 0.5):
    """The same SP branch for the uniform fixed-shape path (the plain-BSA
    dispatch of wan_video_dit.py:470-560, and its variance- / audio-guided forms,
    :637-672): q, k, v [B=1, S_local, num_heads*D] -> x [B, S_local, num_heads*D].
    With a2v_bridge_residual its token norms (all-gathered over SP) drive the
    audio guidance; each rank's variance statistic uses its local heads, as the
    reference's does (bsa_interface.py:989-994).  correction = "rectified" /
    "taylor": the bias-rectified forward (inference; the Taylor split's quantile
    is all-gathered over SP, bias_rectification.py:173-187).  No other collective
    besides the all-to-alls and the norms' all-gather."""
    norms = audio_token_norms(a2v_bridge_residual, full_seq_len)
    kw = dict(sparsity=sparsity, cdf_threshold=cdf_threshold, chunk_3d_shape_q=chunk_3d_shape_q,
              chunk_3d_shape_k=chunk_3d_shape_k, layout="bshd", audio_token_norms=norms,
              audio_gate=audio_gate, audio_boost_gamma=audio_boost_gamma,
              audio_weighted_lambda=audio_weighted_lambda,
              variance_boost_gamma=variance_boost_gamma, correction=correction,
              taylor_alpha_f=taylor_alpha_f)
    x, _ = _sp_self_attention(q, k, v, num_heads, full_seq_len,
                              lambda a, b_, c, ctx: (run_bsa_uniform(a, b_, c, grid_size, **kw), None))
    return x


__all__ = ["dynamic_self_attention", "uniform_self_attention", "audio_token_norms"]
