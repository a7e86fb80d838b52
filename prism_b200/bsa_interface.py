"""Uniform fixed-shape block-sparse attention (drop-in for the reference's
``flash_attn_bsa_3d``, hymm/models/modules/block_sparse_attention/bsa_interface.py:1123-1176).

The shallow half of the DiT under layer-adaptive mode, and every layer without
a dynamic-block trigger, runs this path (wan_video_dit.py:457-468, 470-560):
tokens are rearranged into a global 3D-chunk order (rearrange_THW_to_3d_block,
bsa_interface.py:1105-1109), pooled per chunk, scored, and each q chunk keeps
the key chunks of the hybrid top-k / cumulative-mass rule
(_attention_bsa.forward, bsa_interface.py:600-633); the same sparse attention
kernels as the dynamic path then run on 64-token tiles.

``flash_attn_bsa_3d`` keeps the reference signature: q, k, v [B, H, S, D] in THW
order over ``latent_shape`` (already a multiple of the chunk), optional
``valid_mask`` [S] (True = real token).  ``run_bsa_uniform`` is the uniform
dispatch one level up (pad to the chunk, valid mask, attention, unpad) on
UNPADDED tokens, with the padding and both permutations fused into the
gather / scatter kernels.

Differences from the reference, by design:
* chunk volumes must be multiples of 64 tokens (the training configs use
  4x4x4 = 64; the function default 4x4x8 = 128);
* latent_shape_q must equal latent_shape_k (self-attention; the reference's
  only caller passes the same grid twice);
* without a valid mask the reference pools and scores in bf16; here pooling
  and scores are fp32 always, as the reference does whenever a mask exists.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from . import ops
from .dynamic_block_attention import SparsePlan, _BsaFunction, _check_head_dim, _hsd

_TILE = 64
_PAIR = 128  # the attention kernels work on whole 128-row tile pairs


def _chunk_volume(chunk) -> int:
    return int(chunk[0]) * int(chunk[1]) * int(chunk[2])


def build_uniform_plan(grid, grid_padded, chunk_q, chunk_k, D: int, device, *, sparsity,
                       cdf_threshold, valid_mask: Optional[torch.Tensor] = None) -> SparsePlan:
    """Chunk orders for q and k/v, key validity and selection parameters; no grad.

    grid: the tokens the caller holds (T, H, W); grid_padded: the chunk-multiple
    grid the attention runs on.  Tokens outside ``grid`` are padding, and so are
    tokens with ``valid_mask`` False (valid_mask in padded THW order)."""
    ops.selection_mode(sparsity, cdf_threshold)
    cq, ck = _chunk_volume(chunk_q), _chunk_volume(chunk_k)
    if cq % _TILE or ck % _TILE:
        raise NotImplementedError(
            f"prism_b200 runs chunks of a multiple of {_TILE} tokens, got {cq} and {ck}")
    Tp, Hp, Wp = grid_padded
    seq = Tp * Hp * Wp
    n_rows = int(math.ceil(seq / _PAIR) * _PAIR)
    with torch.no_grad():
        src_q, inv_q = ops.uniform_layout(grid_padded, tuple(chunk_q), n_rows, device)
        if tuple(chunk_q) == tuple(chunk_k):
            src_k, inv_k = src_q, inv_q
        else:
            src_k, inv_k = ops.uniform_layout(grid_padded, tuple(chunk_k), n_rows, device)
        tile_bits, _ = ops.tile_valid(src_k, valid_mask, grid, grid_padded)
    return SparsePlan(grid, grid_padded, dict(src_idx=src_q, inv_idx=inv_q), tile_bits,
                      sparsity, cdf_threshold, 1.0 / (D ** 0.5),
                      layout_k=dict(src_idx=src_k, inv_idx=inv_k),
                      uniform=dict(seq=seq, chunk_q=cq, chunk_k=ck))


def flash_attn_bsa_3d(
    q: torch.Tensor,  # [B, H, Sq, D]
    k: torch.Tensor,  # [B, H, Skv, D]
    v: torch.Tensor,  # [B, H, Skv, D]
    latent_shape_q,
    latent_shape_k,
    sparsity: Optional[float] = 0.875,
    cdf_threshold: Optional[float] = None,
    chunk_3d_shape_q: Sequence[int] = (4, 4, 8),
    chunk_3d_shape_k: Sequence[int] = (4, 4, 8),
    valid_mask: Optional[torch.Tensor] = None,  # [Sq] bool, True = valid token
) -> torch.Tensor:
    """Uniform fixed-shape BSA; returns [B, H, Sq, D] in THW order
    (bsa_interface.py:1123-1176).  Batches are independent heads here."""
    B, Hn, Sq, head_dim_q = q.shape
    _, _, Sk, head_dim_k = k.shape
    assert head_dim_q == head_dim_k
    Tq, Hq, Wq = latent_shape_q
    Tk, Hk, Wk = latent_shape_k
    assert Tq * Hq * Wq == Sq
    assert Tk * Hk * Wk == Sk
    tq, hq, wq = chunk_3d_shape_q
    tk, hk, wk = chunk_3d_shape_k
    assert Tq % tq == 0 and Hq % hq == 0 and Wq % wq == 0
    assert Tk % tk == 0 and Hk % hk == 0 and Wk % wk == 0
    _check_head_dim(head_dim_q)
    if tuple(latent_shape_q) != tuple(latent_shape_k):
        raise NotImplementedError("prism_b200's uniform path is self-attention: "
                                  "latent_shape_q must equal latent_shape_k")
    grid = tuple(int(x) for x in latent_shape_q)
    plan = build_uniform_plan(grid, grid, chunk_3d_shape_q, chunk_3d_shape_k, head_dim_q,
                              q.device, sparsity=sparsity, cdf_threshold=cdf_threshold,
                              valid_mask=valid_mask)
    fold = lambda t: t.reshape(1, B * Hn, t.shape[2], t.shape[3])
    out = _BsaFunction.apply(fold(q), fold(k), fold(v), plan, "bhsd")
    return out.view(B, Hn, Sq, head_dim_q)


def uniform_padded_grid(grid_size, chunk_3d_shape_q, chunk_3d_shape_k) -> Tuple[int, int, int]:
    """Grid padded per axis to the larger chunk extent (wan_video_dit.py:473-481)."""
    m = [max(int(a), int(b)) for a, b in zip(chunk_3d_shape_q, chunk_3d_shape_k)]
    return tuple(int(math.ceil(int(x) / c) * c) for x, c in zip(grid_size, m))


def run_bsa_uniform(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    grid_size: Tuple[int, int, int],
    *,
    sparsity: Optional[float] = 0.875,
    cdf_threshold: Optional[float] = None,
    chunk_3d_shape_q: Sequence[int] = (4, 4, 4),
    chunk_3d_shape_k: Sequence[int] = (4, 4, 4),
    layout: str = "bhsd",
    return_plan: bool = False,
):
    """The plain-BSA branch of the uniform dispatch (wan_video_dit.py:470-560) on
    unpadded tokens: q, k, v [1, H, T*H*W, D] (layout="bhsd") or [1, T*H*W, H, D]
    (layout="bshd").  Pads each axis to the larger chunk extent; the padded
    tokens are masked exactly when padding was needed (valid_mask is None
    otherwise, wan_video_dit.py:485-507).  Output has q's layout."""
    if layout not in ("bhsd", "bshd"):
        raise ValueError("layout must be 'bhsd' or 'bshd'")
    T, H, W = grid_size
    qh = _hsd(q, layout)
    heads, S, D = qh.shape
    assert S == T * H * W, f"sequence {S} != grid {grid_size}"
    assert q.shape[0] == 1, "batch 1"
    _check_head_dim(D)
    gp = uniform_padded_grid(grid_size, chunk_3d_shape_q, chunk_3d_shape_k)
    plan = build_uniform_plan(tuple(grid_size), gp, chunk_3d_shape_q, chunk_3d_shape_k, D,
                              q.device, sparsity=sparsity, cdf_threshold=cdf_threshold)
    out = _BsaFunction.apply(q, k, v, plan, layout)
    return (out, plan) if return_plan else out


__all__ = ["flash_attn_bsa_3d", "run_bsa_uniform", "build_uniform_plan", "uniform_padded_grid"]
