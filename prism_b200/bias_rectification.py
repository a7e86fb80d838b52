"""Bias rectification of the uniform block-sparse path (inference).

Drop-in for hymm/models/modules/block_sparse_attention/bias_rectification.py:

* ``bsa_rectified_sparse_attn`` (:380-446, Rectified SpaAttn): the sparse output
  is rescaled by the mass its selection kept and the dropped chunks come back
  through their pooled values,
  O' = R_n O_spa + (A_pool * unselected) V_cmp, per q chunk;
* ``bsa_taylor_sparse_attn`` (:261-332, LIVEditor): for "flat" q chunks (variance
  of A_pool below the alpha_f quantile over heads, chunks and SP ranks) each
  query also attends to the unselected pooled keys, with log(token count)
  offsets, and the two softmaxes are merged by log-sum-exp (:190-257).

A_pool is the chunk-level softmax of the raw pooled scores over the valid key
chunks.  Inputs are [B, H, S, D] in the 3D-chunk order (rearrange_THW_to_3d_block),
as the correction dispatch of wan_video_dit.py:550-640 passes them; batches fold
into heads (the statistics are per (batch, head) and the quantile runs over all of
them, as the reference's reshape(-1) does).

Everything runs in libprism_bsa.so: the selection and sparse forward of the
uniform path, the chunk statistics (prism_correction_stats), the pooled-key pass
as the forward kernel's key-bias form (prism_bsa_fwd_keybias), the unselected
mass times V_cmp of the rectified form (prism_rectified_contract, fp32 in a fixed
order) and the merges.  Like the reference's fused kernels this path is for
inference: it raises when gradients are required.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import ops
from .bsa_interface import build_uniform_plan
from .dynamic_block_attention import SparsePlan, _hsd, _new_like_layout
from .parallel_states import get_sequence_parallel_state, nccl_info

_PAIR = 128


def global_quantile_across_sp(values: torch.Tensor, q: float) -> torch.Tensor:
    """torch.quantile of the values of every SP rank (_global_quantile_across_sp,
    bias_rectification.py:173-187): each rank holds the same number of values (its
    head shard), gathered in rank order.  A 0-dim fp32 device tensor."""
    flat = values.float().reshape(-1).contiguous()
    if get_sequence_parallel_state() and nccl_info.sp_size > 1:
        parts = [torch.empty_like(flat) for _ in range(nccl_info.sp_size)]
        torch.distributed.all_gather(parts, flat, group=nccl_info.sp_group)
        flat = torch.cat(parts, dim=0)
    return torch.quantile(flat, q)


def corrected_forward(plan: SparsePlan, q_re, k_re, v_re, kind: str, alpha_f: float = 0.5,
                      col_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Selection, sparse forward and the correction on chunk-ordered q / k / v
    [heads, rows, D]; returns the corrected output rows (bf16, chunk order)."""
    if kind not in ("rectified", "taylor"):
        raise ValueError(f"correction must be 'rectified' or 'taylor', got {kind!r}")
    u = plan.uniform
    seq_q, seq_k, cq, ck = u["seq_q"], u["seq_k"], u["chunk_q"], u["chunk_k"]
    tq, tk = cq // 64, ck // 64
    sm = plan.sm_scale
    bits_q, bits_k, pooled = ops.block_select_uniform(
        q_re, k_re, seq_q, seq_k, cq, ck, u["q_bits"], plan.tile_bits, plan.sparsity,
        plan.cdf_threshold, col_scale=col_scale, want_pooled=True)
    plan.bits_q, plan.bits_k = bits_q, bits_k
    # A_pool is taken on the raw scores (the modifier only steers the selection)
    scores = pooled["scores"] if col_scale is None else ops.chunk_scores(pooled["qc"], pooled["kc"])
    o, lse, o_lo = ops.bsa_fwd(q_re, k_re, v_re, bits_q, plan.tile_bits, sm, want_lo=True)
    R, M, nonsel, a_rect = ops.correction_stats(scores, bits_q, plan.tile_bits, tq, tk, sm,
                                                want_nonsel=kind == "taylor",
                                                want_a_rect=kind == "rectified")
    v_cmp = ops.pool_chunks(v_re, seq_k, ck, bits=plan.tile_bits)  # _pool_v, masked mean
    if kind == "rectified":
        o_ncri = ops.rectified_contract(a_rect, v_cmp)  # [heads, nq, D] fp32
        return ops.rectified_apply(o, o_lo, R, o_ncri, seq_q, cq)
    tau = global_quantile_across_sp(M, alpha_f)
    nk = seq_k // ck
    nk_pad = int(math.ceil(nk / _PAIR) * _PAIR)
    k_cmp = ops.rows_to_bf16(pooled["kc"], nk_pad)
    v_cmp16 = ops.rows_to_bf16(v_cmp, nk_pad)
    masks, bits_t = ops.taylor_prep(nonsel, M, tau, q_re.shape[1] // 64, tq, nk, nk_pad // 64)
    bias = ops.key_log_bias(plan.tile_bits, nk, tk, nk_pad, sm)
    o_t, lse_t, o_t_lo = ops.bsa_fwd_keybias(q_re, k_cmp, v_cmp16, bits_t, masks, bias, sm)
    return ops.taylor_merge(o, o_lo, lse, o_t, o_t_lo, lse_t, M, tau, seq_q, cq)


def run_corrected(q, k, v, plan: SparsePlan, layout: str, kind: str, alpha_f: float = 0.5,
                  col_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gather -> corrected_forward -> scatter, for tensors in the plan's layout."""
    _check_inference(q, k, v)
    qh, kh, vh = _hsd(q, layout), _hsd(k, layout), _hsd(v, layout)
    heads, S, D = qh.shape
    with torch.no_grad():
        q_re = ops.gather_rows(qh, plan.grid, plan.grid_padded, plan.src_idx)
        k_re = ops.gather_rows(kh, plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
        v_re = ops.gather_rows(vh, plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
        o_re = corrected_forward(plan, q_re, k_re, v_re, kind, alpha_f, col_scale)
        out, out_hsd = _new_like_layout(heads, S, D, layout, q.dtype, q.device)
        ops.scatter_rows(o_re, plan.grid, plan.grid_padded, plan.inv_idx, out=out_hsd)
    return out


def _check_inference(*ts):
    if torch.is_grad_enabled() and any(t.requires_grad for t in ts):
        raise NotImplementedError(
            "prism_b200 bias rectification is inference-only (as the reference's fused "
            "kernels, bias_rectification_triton.py); run it under torch.no_grad()")


def _modifier_scale(score_modifier, nk: int, device) -> Optional[torch.Tensor]:
    """A multiplicative score modifier broadcastable to [B, H, N_q, N_k] that varies
    only along the key chunks -> [nk] fp32."""
    if score_modifier is None:
        return None
    m = torch.as_tensor(score_modifier, device=device).to(torch.float32)
    if m.numel() == 1:
        return m.reshape(1).expand(nk).contiguous()
    if m.numel() != nk or m.shape[-1] != nk:
        raise NotImplementedError("score_modifier must vary along the key chunks only")
    return m.reshape(nk).contiguous()


def _run_reference_signature(kind, q, k, v, chunk_size_q, chunk_size_k, sparsity, cdf_threshold,
                             sm_scale, alpha_f, kv_valid_mask, q_valid_mask, score_modifier):
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if abs(sm_scale * math.sqrt(D) - 1.0) > 1e-6:
        raise NotImplementedError("sm_scale must be 1/sqrt(head_dim) (the selection uses it too)")
    assert Sq % chunk_size_q == 0 and Sk % chunk_size_k == 0
    if q_valid_mask is not None:
        q_pool = "q"
    elif kv_valid_mask is not None and Sq == Sk:
        q_pool = "k"
    else:
        q_pool = None
    plan = build_uniform_plan((1, 1, Sq), (1, 1, Sq), (1, 1, chunk_size_q), (1, 1, chunk_size_k), D,
                              q.device, sparsity=sparsity, cdf_threshold=cdf_threshold,
                              valid_mask=kv_valid_mask, grid_k=(1, 1, Sk), grid_padded_k=(1, 1, Sk),
                              q_pool=q_pool, valid_mask_q=q_valid_mask)
    scale = _modifier_scale(score_modifier, Sk // chunk_size_k, q.device)
    fold = lambda t: t.reshape(1, B * H, t.shape[2], t.shape[3])
    out = run_corrected(fold(q), fold(k), fold(v), plan, "bhsd", kind, alpha_f, scale)
    return out.view(B, H, Sq, D)


def bsa_rectified_sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, chunk_size_q: int,
                              chunk_size_k: int, sparsity: Optional[float],
                              cdf_threshold: Optional[float], sm_scale: float, *,
                              kv_valid_mask: Optional[torch.Tensor] = None,
                              q_valid_mask: Optional[torch.Tensor] = None,
                              score_modifier: Optional[torch.Tensor] = None,
                              use_triton_inference: bool = True) -> torch.Tensor:
    """Rectified SpaAttn on [B, H, S, D] tensors in the 3D-chunk order
    (bias_rectification.py:380-446).  use_triton_inference is accepted for
    signature compatibility; the CUDA path always runs."""
    return _run_reference_signature("rectified", q, k, v, chunk_size_q, chunk_size_k, sparsity,
                                    cdf_threshold, sm_scale, 0.5, kv_valid_mask, q_valid_mask,
                                    score_modifier)


def bsa_taylor_sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, chunk_size_q: int,
                           chunk_size_k: int, sparsity: Optional[float],
                           cdf_threshold: Optional[float], sm_scale: float, *, alpha_f: float = 0.5,
                           kv_valid_mask: Optional[torch.Tensor] = None,
                           q_valid_mask: Optional[torch.Tensor] = None,
                           score_modifier: Optional[torch.Tensor] = None,
                           use_triton_inference: bool = True) -> torch.Tensor:
    """Taylor (LIVEditor) merge on [B, H, S, D] tensors in the 3D-chunk order
    (bias_rectification.py:261-332)."""
    return _run_reference_signature("taylor", q, k, v, chunk_size_q, chunk_size_k, sparsity,
                                    cdf_threshold, sm_scale, alpha_f, kv_valid_mask, q_valid_mask,
                                    score_modifier)


__all__ = ["bsa_rectified_sparse_attn", "bsa_taylor_sparse_attn", "corrected_forward",
           "run_corrected", "global_quantile_across_sp"]
