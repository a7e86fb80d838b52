"""Dynamic block-shape block-sparse attention (drop-in for the reference's
``hymm/models/modules/block_sparse_attention/dynamic_block_attention.py``).

``flash_attn_bsa_3d_dynamic`` keeps the reference signature and contract
(dynamic_block_attention.py:194-332): q, k, v [1, H, S, D] in THW order,
already padded to the 8x8x8 macro-zone grid, optional audio token norms and
valid mask, optional cached ``shape_ids`` (activation-checkpoint recompute),
output [1, H, S, D] in THW order.

``run_bsa_dynamic`` is the call the DiT makes one level up
(``SelfAttention._run_bsa_dynamic``, wan_video_dit.py:342-432): it takes the
UNPADDED tokens, in either [1, H, S, D] or [1, S, H, D] layout, and fuses the
zero padding, the permutation into tile order and its inverse into the
gather / scatter kernels.

Pipeline per call (all on the current CUDA stream, no host synchronisation):
  zone statistics -> [SP all-reduce] -> shape ids -> permutation / tile maps
  -> gather q,k,v into tile order -> pooled block scores + hybrid selection
  (bitmaps) -> sparse attention forward -> scatter back.
The backward gathers dO, runs the sparse backward and scatters dQ, dK, dV.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import ops
from .dynamic_block_shape import ZONE_SIZE, shapes_from_qkv
from .guidance import guidance_inputs

_TILE = 64  # dynamic_block_attention.py:15


class SparsePlan:
    """Everything the kernels need for one attention call, built without grad.

    ``layout`` orders the queries (src_idx: row -> padded THW token, inv_idx its
    inverse); ``layout_k`` orders keys and values when it differs (the uniform
    path with different q / key chunk shapes).  ``uniform`` = dict(seq, chunk_q,
    chunk_k) selects the uniform path's chunk selection instead of the dynamic
    path's logical-block selection; ``grid_k`` / ``grid_padded_k`` give the keys'
    own grid when it differs from the queries' (cross attention)."""

    def __init__(self, grid, grid_padded, layout, tile_bits, sparsity, cdf_threshold, sm_scale,
                 layout_k=None, uniform=None, grid_k=None, grid_padded_k=None):
        self.grid = tuple(grid)
        self.grid_padded = tuple(grid_padded)
        # keys / values may live on their own grid (cross attention)
        self.grid_k = self.grid if grid_k is None else tuple(grid_k)
        self.grid_padded_k = self.grid_padded if grid_padded_k is None else tuple(grid_padded_k)
        self.layout = layout
        self.src_idx = layout["src_idx"]
        self.inv_idx = layout["inv_idx"]
        lk = layout if layout_k is None else layout_k
        self.src_idx_k = lk["src_idx"]
        self.inv_idx_k = lk["inv_idx"]
        self.uniform = uniform
        self.tile_bits = tile_bits
        self.sparsity = sparsity
        self.cdf_threshold = cdf_threshold
        self.sm_scale = sm_scale
        self.bits_q = None
        self.bits_k = None
        self.seq_capacity = None  # token rows of the outputs' storage (see _new_like_layout)

    def select(self, q_re, k_re, v_re=None):
        """Tile bitmaps (bits_q, bits_k) for tile-ordered q / k (v: the guided
        uniform path's variance statistics)."""
        if self.uniform is not None:
            u = self.uniform
            k_weights = col_scale = None
            if u.get("guidance") is not None:
                k_weights, col_scale = guidance_inputs(self, u["guidance"], v_re)
            return ops.block_select_uniform(q_re, k_re, u["seq_q"], u["seq_k"], u["chunk_q"],
                                            u["chunk_k"], u["q_bits"], self.tile_bits,
                                            self.sparsity, self.cdf_threshold,
                                            k_weights=k_weights, col_scale=col_scale)
        return ops.block_select(q_re, k_re, self.layout, self.tile_bits, self.sparsity,
                                self.cdf_threshold)


def _hsd(x: torch.Tensor, layout: str) -> torch.Tensor:
    """[1,H,S,D] or [1,S,H,D] -> [H,S,D] view with contiguous rows."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x[0] if layout == "bhsd" else x[0].transpose(0, 1)


def _new_like_layout(heads, S, D, layout, dtype, device, capacity=None):
    """A new [1,H,S,D] or [1,S,H,D] tensor and its [H,S,D] view.  capacity (bshd
    only): the storage holds that many token rows and the tensor is its first S
    rows, so a Ulysses exchange can send it without a copy (the rows past S are
    never written or read)."""
    if layout == "bhsd":
        t = torch.empty(1, heads, S, D, dtype=dtype, device=device)
        return t, t[0]
    rows = S if capacity is None else max(int(capacity), S)
    t = torch.empty(1, rows, heads, D, dtype=dtype, device=device)[:, :S]
    return t, t[0].transpose(0, 1)


class _BsaFunction(torch.autograd.Function):
    """Gather -> select -> sparse attention -> scatter, with the matching backward.
    Gradients flow to q, k, v only (selection is non-differentiable, as in the
    reference's no_grad blocks at dynamic_block_attention.py:234, 256 and the
    index tensors of _attention_bsa, bsa_interface.py:597-683)."""

    @staticmethod
    def forward(ctx, q, k, v, plan: SparsePlan, layout: str):
        qh, kh, vh = _hsd(q, layout), _hsd(k, layout), _hsd(v, layout)
        heads, S, D = qh.shape
        Sk = kh.shape[1]
        q_re = ops.gather_rows(qh, plan.grid, plan.grid_padded, plan.src_idx)
        k_re = ops.gather_rows(kh, plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
        v_re = ops.gather_rows(vh, plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
        bits_q, bits_k = plan.select(q_re, k_re, v_re)
        plan.bits_q, plan.bits_k = bits_q, bits_k
        o_re, lse, o_lo = ops.bsa_fwd(q_re, k_re, v_re, bits_q, plan.tile_bits, plan.sm_scale,
                                      want_lo=True)
        out, out_hsd = _new_like_layout(heads, S, D, layout, q.dtype, q.device, plan.seq_capacity)
        ops.scatter_rows(o_re, plan.grid, plan.grid_padded, plan.inv_idx, out=out_hsd)
        ctx.save_for_backward(q_re, k_re, v_re, o_re, o_lo, lse, bits_q, bits_k)
        ctx.plan = plan
        ctx.layout = layout
        ctx.shape = (heads, S, Sk, D)
        return out

    @staticmethod
    def backward(ctx, dout):
        q_re, k_re, v_re, o_re, o_lo, lse, bits_q, bits_k = ctx.saved_tensors
        plan = ctx.plan
        layout = ctx.layout
        heads, S, Sk, D = ctx.shape
        do_re = ops.gather_rows(_hsd(dout, layout), plan.grid, plan.grid_padded, plan.src_idx)
        dq_re, dk_re, dv_re = ops.bsa_bwd(q_re, k_re, v_re, o_re, do_re, lse, bits_q, bits_k,
                                          plan.tile_bits, plan.sm_scale, o_lo=o_lo)
        grads = []
        for g_re, is_k in ((dq_re, False), (dk_re, True), (dv_re, True)):
            g, g_hsd = _new_like_layout(heads, Sk if is_k else S, D, layout, dout.dtype, dout.device,
                                        plan.seq_capacity)
            if is_k:
                ops.scatter_rows(g_re, plan.grid_k, plan.grid_padded_k, plan.inv_idx_k, out=g_hsd)
            else:
                ops.scatter_rows(g_re, plan.grid, plan.grid_padded, plan.inv_idx, out=g_hsd)
            grads.append(g)
        return grads[0], grads[1], grads[2], None, None


_DynBsaFunction = _BsaFunction


def _check_head_dim(D: int):
    """The reference's head-dim contract (bsa_interface.py:604-605).  16 and 32 run on the
    D = 64 kernels with zero columns (ops.bsa_fwd / ops.bsa_bwd); 256 is not built."""
    assert D in {16, 32, 64, 128, 256}, "head dim must be one of 16, 32, 64, 128, 256"
    if D == 256:
        raise NotImplementedError("prism_b200 attention kernels take head_dim 16, 32, 64 or 128, got 256")


def build_plan(q_hsd, k_hsd, v_hsd, grid, grid_padded, *, method, sparsity, cdf_threshold,
               audio_token_norms=None, valid_mask=None, lambda_a=0.5, tau_128=0.15,
               lambda_128=1.0, shape_ids=None, sp_live_ranks=None):
    """Shape ids (unless given), permutation, tile maps and key validity; no grad.
    sp_live_ranks: SP ranks that contribute zone statistics (default: all)."""
    ops.selection_mode(sparsity, cdf_threshold)
    D = q_hsd.shape[-1]
    with torch.no_grad():
        if shape_ids is None:
            shape_ids = shapes_from_qkv(v_hsd, grid, grid_padded, method,
                                        audio_norms=audio_token_norms, valid_mask=valid_mask,
                                        lambda_a=lambda_a, tau_128=tau_128, lambda_128=lambda_128,
                                        sp_live_ranks=sp_live_ranks)
        layout = ops.build_layout(shape_ids, grid_padded)
        tile_bits, _ = ops.tile_valid(layout["src_idx"], valid_mask, grid, grid_padded)
    plan = SparsePlan(grid, grid_padded, layout, tile_bits, sparsity, cdf_threshold,
                      1.0 / (D ** 0.5))
    return plan, shape_ids


def flash_attn_bsa_3d_dynamic(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    grid_padded: Tuple[int, int, int],
    *,
    method: str,
    sparsity: Optional[float] = 0.9375,
    cdf_threshold: Optional[float] = None,
    audio_token_norms: Optional[torch.Tensor] = None,
    valid_mask: Optional[torch.Tensor] = None,
    lambda_a: float = 0.5,
    tau_128: float = 0.15,
    lambda_128: float = 1.0,
    shape_ids: Optional[torch.Tensor] = None,
    return_shape_ids: bool = False,
):
    """Dynamic-block-shape BSA for video self-attention. Returns [B,H,S,D] THW order.

    Same contract as the reference (dynamic_block_attention.py:194-332):
    shape_ids, if given, skips the shape choice (checkpoint recompute);
    return_shape_ids returns it as well."""
    B, Hn, S, D = q.shape
    T, H, W = grid_padded
    assert T * H * W == S
    assert T % ZONE_SIZE == 0 and H % ZONE_SIZE == 0 and W % ZONE_SIZE == 0
    assert B == 1, "the dynamic path takes shape statistics from v[0] (batch 1)"
    _check_head_dim(D)
    if shape_ids is None and method not in ("ivpq", "penalty"):
        raise ValueError(f"unknown dynamic-block method: {method!r}")
    plan, shape_ids = build_plan(
        _hsd(q, "bhsd"), _hsd(k, "bhsd"), _hsd(v, "bhsd"), grid_padded, grid_padded,
        method=method, sparsity=sparsity, cdf_threshold=cdf_threshold,
        audio_token_norms=audio_token_norms, valid_mask=valid_mask, lambda_a=lambda_a,
        tau_128=tau_128, lambda_128=lambda_128, shape_ids=shape_ids)
    out = _DynBsaFunction.apply(q, k, v, plan, "bhsd")
    if return_shape_ids:
        return out, shape_ids
    return out


def run_bsa_dynamic(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    grid_size: Tuple[int, int, int],
    *,
    method: str = "ivpq",
    sparsity: Optional[float] = 0.9375,
    cdf_threshold: Optional[float] = None,
    audio_token_norms: Optional[torch.Tensor] = None,
    lambda_a: float = 0.5,
    tau_128: float = 0.15,
    lambda_128: float = 1.0,
    shape_ids: Optional[torch.Tensor] = None,
    return_shape_ids: bool = False,
    layout: str = "bhsd",
    return_plan: bool = False,
    seq_capacity: Optional[int] = None,
    sp_live_ranks: Optional[int] = None,
):
    """``SelfAttention._run_bsa_dynamic`` (wan_video_dit.py:342-432) on unpadded
    tokens: q, k, v [1, H, T*H*W, D] (layout="bhsd") or [1, T*H*W, H, D]
    (layout="bshd"), audio_token_norms [T*H*W] or None.  Padding to the zone
    grid, the valid mask and the unpad are implicit.  Output has q's layout.
    seq_capacity (bshd): the output and the input gradients are the first
    T*H*W rows of buffers of that many rows (a Ulysses exchange sends them
    without a copy); sp_live_ranks: SP ranks whose zone statistics are averaged
    (ranks holding only padding heads contribute zeros)."""
    if layout not in ("bhsd", "bshd"):
        raise ValueError("layout must be 'bhsd' or 'bshd'")
    T, H, W = grid_size
    qh = _hsd(q, layout)
    heads, S, D = qh.shape
    assert S == T * H * W, f"sequence {S} != grid {grid_size}"
    assert q.shape[0] == 1, "batch 1"
    _check_head_dim(D)
    gp = ops.padded_grid(grid_size)
    plan, shape_ids = build_plan(
        qh, _hsd(k, layout), _hsd(v, layout), grid_size, gp, method=method, sparsity=sparsity,
        cdf_threshold=cdf_threshold, audio_token_norms=audio_token_norms, valid_mask=None,
        lambda_a=lambda_a, tau_128=tau_128, lambda_128=lambda_128, shape_ids=shape_ids,
        sp_live_ranks=sp_live_ranks)
    if layout == "bshd":
        plan.seq_capacity = seq_capacity
    out = _DynBsaFunction.apply(q, k, v, plan, layout)
    res = [out]
    if return_shape_ids:
        res.append(shape_ids)
    if return_plan:
        res.append(plan)
    return res[0] if len(res) == 1 else tuple(res)


__all__ = ["flash_attn_bsa_3d_dynamic", "run_bsa_dynamic", "build_plan", "SparsePlan"]
