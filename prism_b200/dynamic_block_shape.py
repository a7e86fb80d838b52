"""Per-zone anisotropic block-shape choice on the GPU.

Same public names and semantics as the reference module
``hymm/models/modules/block_sparse_attention/dynamic_block_shape.py``:
candidate shapes (:6-31), ``compute_effective_gradient`` (:248-301),
``select_shapes_ivpq`` / ``select_shapes_penalty`` (:303-355) and
``select_zone_shapes`` (:358-391).  The zone statistics and the shape choice
run as two CUDA kernels; the SP average of the packed statistics
(``_maybe_sp_average``, :132-151) is one NCCL all-reduce between them.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops
from .parallel_states import get_sequence_parallel_state, nccl_info

CANDIDATE_SHAPES_64: List[Tuple[int, int, int]] = [
    (4, 4, 4), (8, 2, 4), (8, 4, 2), (2, 4, 8), (2, 8, 4), (4, 2, 8), (4, 8, 2),
]
CANDIDATE_SHAPES_128: List[Tuple[int, int, int]] = [
    (2, 8, 8), (8, 2, 8), (8, 8, 2), (4, 4, 8), (4, 8, 4), (8, 4, 4),
]
ALL_CANDIDATE_SHAPES = CANDIDATE_SHAPES_64 + CANDIDATE_SHAPES_128
NUM_CANDIDATES_64 = len(CANDIDATE_SHAPES_64)
NUM_CANDIDATES = len(ALL_CANDIDATE_SHAPES)
ZONE_SIZE = 8


def _maybe_sp_average(packed: torch.Tensor, sp_reduce: bool = True,
                      live_ranks: Optional[int] = None) -> torch.Tensor:
    """Average of the packed zone means over the SP group (dynamic_block_shape.py:
    132-151): one SUM all-reduce, divided by the number of ranks that hold real
    heads (``live_ranks``, default every rank -- the reference's AVG).  A rank
    holding only padding heads joins the collective with zeros; the reference's
    such rank would not join at all (its peers would wait forever), so dividing
    by the live ranks keeps the average that of the ranks with data.  No
    try/except: a rank that skipped the collective must fail loudly."""
    if not sp_reduce or (not get_sequence_parallel_state()) or nccl_info.sp_size <= 1:
        return packed
    dist.all_reduce(packed, op=dist.ReduceOp.SUM, group=nccl_info.sp_group)
    packed /= float(nccl_info.sp_size if live_ranks is None else live_ranks)
    return packed


def zone_statistics(v_hsd: torch.Tensor, grid, grid_padded, valid_mask=None, audio_norms=None,
                    sp_reduce: bool = True, sp_live_ranks: Optional[int] = None):
    """Head-averaged V zone means (SP-averaged) + axis validity + audio zone means."""
    packed, axis_valid, audio = ops.zone_stats(v_hsd, grid, grid_padded, valid_mask, audio_norms)
    packed = _maybe_sp_average(packed, sp_reduce, sp_live_ranks)
    return packed, axis_valid, audio


def compute_effective_gradient(v_headavg_thw_d: torch.Tensor, audio_norms_thw: Optional[torch.Tensor],
                               ZT: int, ZH: int, ZW: int, lambda_a: float = 0.5,
                               valid_mask_thw: Optional[torch.Tensor] = None,
                               sp_reduce: bool = True):
    """(g [Nz,3], rho [Nz]) from a head-averaged V [T,H,W,D] (bf16)."""
    T, H, W, D = v_headavg_thw_d.shape
    v = v_headavg_thw_d.reshape(1, T * H * W, D)
    grid = (T, H, W)
    packed, av, audio = zone_statistics(v, grid, grid, valid_mask_thw, audio_norms_thw, sp_reduce)
    _, g, rho = ops.shape_select(packed, av, audio, audio_norms_thw is not None, "ivpq", lambda_a,
                                 want_diag=True)
    return g, rho


def select_zone_shapes(v_headavg_thw_d: torch.Tensor, audio_norms_thw: Optional[torch.Tensor],
                       grid_padded: Tuple[int, int, int], method: str, lambda_a: float = 0.5,
                       tau_128: float = 0.15, lambda_128: float = 1.0,
                       valid_mask_thw: Optional[torch.Tensor] = None,
                       sp_reduce: bool = True) -> torch.Tensor:
    """features -> shape id per zone, int64 [num_zones] (dynamic_block_shape.py:358-391)."""
    T, H, W = grid_padded
    assert T % ZONE_SIZE == 0 and H % ZONE_SIZE == 0 and W % ZONE_SIZE == 0, (
        f"grid {grid_padded} must be multiple of zone size {ZONE_SIZE}")
    if method not in ("ivpq", "penalty"):
        raise ValueError(f"unknown dynamic-block method: {method!r}")
    D = v_headavg_thw_d.shape[-1]
    v = v_headavg_thw_d.reshape(1, T * H * W, D)
    packed, av, audio = zone_statistics(v, grid_padded, grid_padded, valid_mask_thw,
                                        audio_norms_thw, sp_reduce)
    return ops.shape_select(packed, av, audio, audio_norms_thw is not None, method, lambda_a,
                            tau_128, lambda_128)


def shapes_from_qkv(v_hsd: torch.Tensor, grid, grid_padded, method: str, audio_norms=None,
                    valid_mask=None, lambda_a=0.5, tau_128=0.15, lambda_128=1.0,
                    sp_reduce: bool = True, sp_live_ranks: Optional[int] = None) -> torch.Tensor:
    """Shape ids straight from the per-head V of the attention call (fuses the
    head average of dynamic_block_attention.py:236 into the zone statistics)."""
    if method not in ("ivpq", "penalty"):
        raise ValueError(f"unknown dynamic-block method: {method!r}")
    packed, av, audio = zone_statistics(v_hsd, grid, grid_padded, valid_mask, audio_norms, sp_reduce,
                                        sp_live_ranks)
    return ops.shape_select(packed, av, audio, audio_norms is not None, method, lambda_a, tau_128,
                            lambda_128)


__all__ = [
    "CANDIDATE_SHAPES_64", "CANDIDATE_SHAPES_128", "ALL_CANDIDATE_SHAPES", "NUM_CANDIDATES_64",
    "NUM_CANDIDATES", "ZONE_SIZE", "compute_effective_gradient", "select_zone_shapes",
    "shapes_from_qkv", "zone_statistics",
]
