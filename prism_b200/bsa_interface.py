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

``flash_attn_bsa_3d_variance_guided`` / ``flash_attn_bsa_3d_audio_guided``
(bsa_interface.py:1179-1260, 1395-1501) add a per-key-chunk score factor
(prism_b200/guidance.py) to the same selection.

``flash_attn_bsa_cross`` (bsa_interface.py:1276-1392) is the cross-modal form
(3D video and/or 1D audio queries and keys, each side padded to its own chunk)
on the same plan and kernels.

Differences from the reference, by design:
* chunk volumes must be multiples of 64 tokens (the training configs use
  4x4x4 = 64; the function default 4x4x8 = 128; 1D chunks default to 64);
* without a valid mask the reference pools and scores in bf16; here pooling
  and scores are fp32 always, as the reference does whenever a mask exists.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch

from . import ops
from .dynamic_block_attention import SparsePlan, _BsaFunction, _check_head_dim, _hsd
from .guidance import guidance_inputs, make_guidance

_TILE = 64
_PAIR = 128  # the attention kernels work on whole 128-row tile pairs


def _chunk_volume(chunk) -> int:
    return int(chunk[0]) * int(chunk[1]) * int(chunk[2])


def _rows(seq: int) -> int:
    return int(math.ceil(seq / _PAIR) * _PAIR)


def build_uniform_plan(grid, grid_padded, chunk_q, chunk_k, D: int, device, *, sparsity,
                       cdf_threshold, valid_mask: Optional[torch.Tensor] = None,
                       grid_k=None, grid_padded_k=None, q_pool: Optional[str] = "k",
                       valid_mask_q: Optional[torch.Tensor] = None) -> SparsePlan:
    """Chunk orders for q and k/v, key validity and selection parameters; no grad.

    grid: the query tokens the caller holds (T, H, W); grid_padded: the chunk-multiple
    grid the attention runs on.  grid_k / grid_padded_k: the keys' grids (default: the
    queries').  Key tokens outside grid_k are padding, and so are keys with valid_mask
    False (padded THW order of the key grid).  q_pool selects the rows the q pooling
    counts: "k" = the key mask at the same positions (the reference's behaviour for
    q and k of one sequence, bsa_interface.py:609-610), "q" = the queries' own
    validity (grid plus valid_mask_q), None = every row."""
    ops.selection_mode(sparsity, cdf_threshold)
    cq, ck = _chunk_volume(chunk_q), _chunk_volume(chunk_k)
    if cq % _TILE or ck % _TILE:
        raise NotImplementedError(
            f"prism_b200 runs chunks of a multiple of {_TILE} tokens, got {cq} and {ck}")
    grid_k = tuple(grid) if grid_k is None else tuple(grid_k)
    grid_padded_k = tuple(grid_padded) if grid_padded_k is None else tuple(grid_padded_k)
    seq_q = int(math.prod(grid_padded))
    seq_k = int(math.prod(grid_padded_k))
    with torch.no_grad():
        src_q, inv_q = ops.uniform_layout(grid_padded, tuple(chunk_q), _rows(seq_q), device)
        if tuple(chunk_q) == tuple(chunk_k) and grid_padded_k == tuple(grid_padded):
            src_k, inv_k = src_q, inv_q
        else:
            src_k, inv_k = ops.uniform_layout(grid_padded_k, tuple(chunk_k), _rows(seq_k), device)
        tile_bits, _ = ops.tile_valid(src_k, valid_mask, grid_k, grid_padded_k)
        if q_pool == "k":
            if seq_q != seq_k:
                raise ValueError("q pooled under the key mask needs equal q and k lengths")
            q_bits = tile_bits
        elif q_pool == "q":
            q_bits, _ = ops.tile_valid(src_q, valid_mask_q, grid, grid_padded)
        else:
            q_bits = None
    return SparsePlan(grid, grid_padded, dict(src_idx=src_q, inv_idx=inv_q), tile_bits,
                      sparsity, cdf_threshold, 1.0 / (D ** 0.5),
                      layout_k=dict(src_idx=src_k, inv_idx=inv_k),
                      uniform=dict(seq_q=seq_q, seq_k=seq_k, chunk_q=cq, chunk_k=ck, q_bits=q_bits),
                      grid_k=grid_k, grid_padded_k=grid_padded_k)


def _bsa_3d(q, k, v, latent_shape_q, latent_shape_k, sparsity, cdf_threshold, chunk_3d_shape_q,
            chunk_3d_shape_k, valid_mask, guidance_kw=None):
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
    gq = tuple(int(x) for x in latent_shape_q)
    gk = tuple(int(x) for x in latent_shape_k)
    if valid_mask is not None:
        assert valid_mask.numel() == Sk, "valid_mask masks the keys: [Skv] elements"
    q_pool = "k" if (valid_mask is not None and Sq == Sk) else None
    plan = build_uniform_plan(gq, gq, chunk_3d_shape_q, chunk_3d_shape_k, head_dim_q, q.device,
                              sparsity=sparsity, cdf_threshold=cdf_threshold,
                              valid_mask=valid_mask, grid_k=gk, grid_padded_k=gk, q_pool=q_pool)
    if guidance_kw is not None:
        if B != 1:
            raise NotImplementedError("guided selection runs batch 1 (the reference's statistics "
                                      "read batch 0, bsa_interface.py:1033)")
        nk = Sk // _chunk_volume(chunk_3d_shape_k)
        plan.uniform["guidance"] = make_guidance(chunk_3d_shape_k, n_chunks_k=nk, device=q.device,
                                                 **guidance_kw)
    fold = lambda t: t.reshape(1, B * Hn, t.shape[2], t.shape[3])
    out = _BsaFunction.apply(fold(q), fold(k), fold(v), plan, "bhsd")
    return out.view(B, Hn, Sq, head_dim_q)


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
    valid_mask: Optional[torch.Tensor] = None,  # [Skv] bool, True = valid token
) -> torch.Tensor:
    """Uniform fixed-shape BSA; returns [B, H, Sq, D] in THW order
    (bsa_interface.py:1123-1176).  Batches are independent heads here.  valid_mask
    masks the keys (rearranged with the key chunk, :1160-1162); q is pooled under it
    when q and k have the same length (:609-610), else over every row."""
    return _bsa_3d(q, k, v, latent_shape_q, latent_shape_k, sparsity, cdf_threshold,
                   chunk_3d_shape_q, chunk_3d_shape_k, valid_mask)


def flash_attn_bsa_3d_variance_guided(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    latent_shape_q,
    latent_shape_k,
    variance_boost_gamma: float = 1.0,
    sparsity: Optional[float] = 0.875,
    cdf_threshold: Optional[float] = None,
    chunk_3d_shape_q: Sequence[int] = (4, 4, 4),
    chunk_3d_shape_k: Sequence[int] = (4, 4, 4),
    valid_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """flash_attn_bsa_3d with each key chunk's scores scaled by 1 + gamma * rho_j,
    rho the channel-variance density of V (bsa_interface.py:1179-1260)."""
    return _bsa_3d(q, k, v, latent_shape_q, latent_shape_k, sparsity, cdf_threshold,
                   chunk_3d_shape_q, chunk_3d_shape_k, valid_mask,
                   guidance_kw=dict(variance_gamma=float(variance_boost_gamma)))


def flash_attn_bsa_3d_audio_guided(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    latent_shape_q,
    latent_shape_k,
    audio_token_norms: Optional[torch.Tensor] = None,
    audio_gate_value=None,
    audio_boost_gamma=None,
    sparsity: Optional[float] = 0.875,
    cdf_threshold: Optional[float] = None,
    chunk_3d_shape_q: Sequence[int] = (4, 4, 4),
    chunk_3d_shape_k: Sequence[int] = (4, 4, 4),
    valid_mask: Optional[torch.Tensor] = None,
    audio_weighted_lambda: float = 0.0,
    score_modifier: Optional[torch.Tensor] = None,
    variance_boost_gamma: float = 0.0,
) -> torch.Tensor:
    """flash_attn_bsa_3d with audio-saliency score modulation
    (bsa_interface.py:1395-1501): scores of key chunk j scaled by
    1 + gamma_a * (g * S_j + (1 - g) / N) [+ gamma_v * rho_j] [+ score_modifier_j],
    S the block saliency of audio_token_norms (per key token, THW order; None = no
    audio term), keys pooled with the audio weights when audio_weighted_lambda > 0
    (Path B)."""
    return _bsa_3d(q, k, v, latent_shape_q, latent_shape_k, sparsity, cdf_threshold,
                   chunk_3d_shape_q, chunk_3d_shape_k, valid_mask,
                   guidance_kw=dict(variance_gamma=float(variance_boost_gamma or 0.0),
                                    audio_token_norms=audio_token_norms,
                                    audio_gate=audio_gate_value, audio_gamma=audio_boost_gamma,
                                    audio_weighted_lambda=float(audio_weighted_lambda or 0.0),
                                    score_modifier=score_modifier))


def _structure_grid(structure: str, n_tokens: int, grid_size, chunk_1d: int, chunk_3d):
    """(grid, padded grid, chunk) of one side of flash_attn_bsa_cross: "3d" = the
    latent grid padded per axis to the chunk (default 4x4x4), "1d" = a (1, 1, S) grid
    padded to chunk_1d tokens (_pad_1d_for_bsa, bsa_interface.py:1263-1273)."""
    if structure == "3d":
        assert grid_size is not None
        grid = tuple(int(x) for x in grid_size)
        assert grid[0] * grid[1] * grid[2] == n_tokens
        chunk = tuple(int(x) for x in (chunk_3d or (4, 4, 4)))
        padded = tuple(int(math.ceil(g / c) * c) for g, c in zip(grid, chunk))
        return grid, padded, chunk
    if structure == "1d":
        if chunk_1d % _TILE:
            raise NotImplementedError(
                f"prism_b200 runs chunks of a multiple of {_TILE} tokens, got {chunk_1d}")
        grid = (1, 1, int(n_tokens))
        return grid, (1, 1, int(math.ceil(n_tokens / chunk_1d) * chunk_1d)), (1, 1, int(chunk_1d))
    raise ValueError(f"structure must be '3d' or '1d', got {structure!r}")


def build_cross_plan(q_structure: str, k_structure: str, Sq: int, Sk: int, D: int, device, *,
                     q_grid_size=None, k_grid_size=None, sparsity=0.875, cdf_threshold=None,
                     chunk_size_q: int = 64, chunk_size_k: int = 64, chunk_3d_shape_q=None,
                     chunk_3d_shape_k=None) -> SparsePlan:
    """The plan of flash_attn_bsa_cross: each side's grid, padding and chunk order;
    a padded q side pools over its real rows, else q pools under the key mask when
    the lengths agree, else over every row (bsa_interface.py:606-611)."""
    gq, gpq, cq = _structure_grid(q_structure, Sq, q_grid_size, chunk_size_q, chunk_3d_shape_q)
    gk, gpk, ck = _structure_grid(k_structure, Sk, k_grid_size, chunk_size_k, chunk_3d_shape_k)
    seq_q, seq_k = math.prod(gpq), math.prod(gpk)
    if gq != gpq:
        q_pool = "q"
    elif gk != gpk and seq_q == seq_k:
        q_pool = "k"
    else:
        q_pool = None
    return build_uniform_plan(gq, gpq, cq, ck, D, device, sparsity=sparsity,
                              cdf_threshold=cdf_threshold, grid_k=gk, grid_padded_k=gpk,
                              q_pool=q_pool)


def flash_attn_bsa_cross(
    q: torch.Tensor,  # [B, H, Sq, D]
    k: torch.Tensor,  # [B, H, Sk, D]
    v: torch.Tensor,  # [B, H, Sk, D]
    q_structure: str,
    k_structure: str,
    q_grid_size=None,
    k_grid_size=None,
    sparsity: Optional[float] = 0.875,
    cdf_threshold: Optional[float] = None,
    chunk_size_q: int = 64,
    chunk_size_k: int = 64,
    chunk_3d_shape_q=None,
    chunk_3d_shape_k=None,
) -> torch.Tensor:
    """Cross-modal BSA with 3D (video grid) or 1D (audio sequence) queries and keys
    (bsa_interface.py:1276-1392).  Each side is padded to its chunk, a padded q side
    pools q over its real rows and a padded k side masks its padding keys; returns
    [B, H, Sq, D] on the queries' own (unpadded) token order."""
    B, Hn, Sq, D = q.shape
    Sk = k.shape[2]
    assert k.shape[3] == D and v.shape[2] == Sk
    _check_head_dim(D)
    plan = build_cross_plan(q_structure, k_structure, Sq, Sk, D, q.device,
                            q_grid_size=q_grid_size, k_grid_size=k_grid_size, sparsity=sparsity,
                            cdf_threshold=cdf_threshold, chunk_size_q=chunk_size_q,
                            chunk_size_k=chunk_size_k, chunk_3d_shape_q=chunk_3d_shape_q,
                            chunk_3d_shape_k=chunk_3d_shape_k)
    fold = lambda t: t.reshape(1, B * Hn, t.shape[2], t.shape[3])
    out = _BsaFunction.apply(fold(q), fold(k), fold(v), plan, "bhsd")
    return out.view(B, Hn, Sq, D)


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
    audio_token_norms: Optional[torch.Tensor] = None,
    audio_gate=None,
    audio_boost_gamma=None,
    audio_weighted_lambda: float = 0.0,
    variance_boost_gamma: float = 0.0,
    correction: Optional[str] = None,
    taylor_alpha_f: float = 0.5,
):
    """The uniform dispatch (wan_video_dit.py:470-560, 637-672) on unpadded tokens:
    q, k, v [1, H, T*H*W, D] (layout="bhsd") or [1, T*H*W, H, D] (layout="bshd").
    Pads each axis to the larger chunk extent; the padded tokens are masked exactly
    when padding was needed (valid_mask is None otherwise, wan_video_dit.py:485-507).
    Guidance as the dispatch picks it: variance_boost_gamma > 0 = the variance
    term; audio_token_norms [T*H*W] (unpadded) = the audio-guided path with gate
    audio_gate, gain audio_boost_gamma and Path B weight audio_weighted_lambda
    (zero-padded norms, wan_video_dit.py:299-306).  correction = "rectified" or
    "taylor" runs the bias-rectified forward instead (inference only, the
    correction dispatch of wan_video_dit.py:550-640: the guidance then only scales
    the selection's scores and Path B is ignored, as there).  Output has q's
    layout."""
    if layout not in ("bhsd", "bshd"):
        raise ValueError("layout must be 'bhsd' or 'bshd'")
    T, H, W = grid_size
    qh = _hsd(q, layout)
    heads, S, D = qh.shape
    assert S == T * H * W, f"sequence {S} != grid {grid_size}"
    assert q.shape[0] == 1, "batch 1"
    _check_head_dim(D)
    gp = uniform_padded_grid(grid_size, chunk_3d_shape_q, chunk_3d_shape_k)
    padded = tuple(gp) != tuple(grid_size)
    plan = build_uniform_plan(tuple(grid_size), gp, chunk_3d_shape_q, chunk_3d_shape_k, D,
                              q.device, sparsity=sparsity, cdf_threshold=cdf_threshold,
                              q_pool="k" if padded else None)
    if variance_boost_gamma or audio_token_norms is not None:
        nk = plan.uniform["seq_k"] // plan.uniform["chunk_k"]
        plan.uniform["guidance"] = make_guidance(
            chunk_3d_shape_k, variance_gamma=float(variance_boost_gamma or 0.0),
            audio_token_norms=audio_token_norms, audio_gate=audio_gate,
            audio_gamma=audio_boost_gamma, audio_weighted_lambda=float(audio_weighted_lambda or 0.0),
            n_chunks_k=nk, device=q.device)
    if correction is not None:
        from .bias_rectification import run_corrected
        scale = None
        g = plan.uniform.pop("guidance", None)
        if g is not None:
            g = dict(g, lambda_w=0.0)
            with torch.no_grad():
                v_re = ops.gather_rows(_hsd(v, layout), plan.grid_k, plan.grid_padded_k,
                                       plan.src_idx_k) if g["variance_gamma"] > 0 else None
                _, scale = guidance_inputs(plan, g, v_re)
        out = run_corrected(q, k, v, plan, layout, correction, taylor_alpha_f, scale)
        return (out, plan) if return_plan else out
    out = _BsaFunction.apply(q, k, v, plan, layout)
    return (out, plan) if return_plan else out


__all__ = ["flash_attn_bsa_3d", "flash_attn_bsa_3d_variance_guided", "flash_attn_bsa_3d_audio_guided",
           "flash_attn_bsa_cross", "run_bsa_uniform", "build_uniform_plan", "build_cross_plan",
           "uniform_padded_grid"]
