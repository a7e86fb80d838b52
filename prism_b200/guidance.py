"""Score guidance of the uniform block-sparse path.

The reference modulates the chunk-level scores before the selection with a
per-key-chunk factor (hymm/models/modules/block_sparse_attention/bsa_interface.py):

* ``flash_attn_bsa_3d_variance_guided`` (:1179-1260): score *= 1 + gamma * rho_j,
  rho = ``compute_channel_variance_density`` (:973-1062) of V;
* ``flash_attn_bsa_3d_audio_guided`` (:1395-1501, autograd function :686-828):
  score *= 1 + gamma_a * (g * S_j + (1 - g) / N) [+ gamma_v * rho_j] [+ modifier_j]
  with S = ``compute_block_audio_saliency`` (:1065-1102) of the a2v norms, and
  optionally the keys pooled with ``audio_weighted_mean_pooling_compression``
  (:902-970, "Path B") instead of the masked mean.

The sparse attention itself is unchanged.  Here every statistic is a kernel of
libprism_bsa.so on the chunk-ordered keys the attention already gathered; the
factor enters the selection as ``col_scale`` and Path B as ``k_weights`` of
``prism_block_select_uniform``.  The scalar gates g (``compute_audio_spatial_
concentration_gate`` :866-899, ``compute_timestep_reliability_gate`` :831-863)
stay device tensors.

The helpers below keep the reference's names and arguments (batch 1, the
[B, H, S, D] tensors already in 3D-chunk order).  Statistics are fp32 in every
case; the reference computes them in the input dtype and rounds rho and the
factor to it (``rho.to(q.dtype)``), so with bf16 inputs its selection can
differ from this one where two chunk scores are within bf16 rounding.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import ops


def _valid_bits(valid_mask: Optional[torch.Tensor], n: int, device) -> Optional[torch.Tensor]:
    """[n] bool validity -> row-validity words (64 rows per word); None stays None."""
    if valid_mask is None:
        return None
    rows = int(math.ceil(n / 64) * 64)
    src = torch.arange(rows, dtype=torch.int32, device=device)
    bits, _ = ops.tile_valid(src, valid_mask.reshape(-1).to(device=device, dtype=torch.bool),
                             (1, 1, n), (1, 1, rows))
    return bits


def _pad_rows(n: int, chunk: int) -> int:
    return int(math.ceil(n / chunk) * chunk)


def compute_channel_variance_density(x: torch.Tensor, block_size: int, bt: int, bh: int, bw: int,
                                     valid_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """rho [num_blocks] fp32 in [0, 1] of V x [1, H, S, D] (bf16, 3D-chunk order)
    (bsa_interface.py:973-1062)."""
    B, H, S, D = x.shape
    if B != 1:
        raise NotImplementedError("batch 1 (the reference averages x[0])")
    if x.dtype != torch.bfloat16:
        raise TypeError("compute_channel_variance_density expects bf16 V")
    assert block_size == bt * bh * bw and S % block_size == 0
    xh = x[0] if x[0].is_contiguous() else x[0].contiguous()
    return ops.variance_density(xh, S, (bt, bh, bw), _valid_bits(valid_mask, S, x.device))


def compute_block_audio_saliency(token_norms: torch.Tensor, chunk_size: int,
                                 valid_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-block audio saliency [N_blocks] fp32 (bsa_interface.py:1065-1102).  A
    ragged tail is zero-padded (counted as tokens when there is no mask, as the
    reference's F.pad does)."""
    S = token_norms.numel()
    Sp = _pad_rows(S, chunk_size)
    a = torch.zeros(Sp, dtype=torch.float32, device=token_norms.device)
    a[:S] = token_norms.reshape(-1)
    vm = None
    if valid_mask is not None:
        vm = torch.zeros(Sp, dtype=torch.bool, device=token_norms.device)
        vm[:S] = valid_mask.reshape(-1)
    return ops.audio_saliency(a, Sp, chunk_size, _valid_bits(vm, Sp, a.device))


def audio_weighted_mean_pooling_compression(x: torch.Tensor, block_size: int,
                                            token_norms: torch.Tensor,
                                            valid_mask: Optional[torch.Tensor] = None,
                                            lambda_w: float = 1.0) -> torch.Tensor:
    """Audio-weighted chunk means [B, H, N_blocks, D] fp32 of x [B, H, S, D] bf16
    (Path B, bsa_interface.py:902-970)."""
    B, H, S, D = x.shape
    if x.dtype != torch.bfloat16:
        raise TypeError("audio_weighted_mean_pooling_compression expects bf16")
    Sp = _pad_rows(S, block_size)
    xh = x.reshape(B * H, S, D)
    if Sp != S:
        xh = torch.nn.functional.pad(xh, (0, 0, 0, Sp - S))
    xh = xh.contiguous()
    a = torch.zeros(Sp, dtype=torch.float32, device=x.device)
    a[:S] = token_norms.reshape(-1)
    vm = None
    if valid_mask is not None:
        vm = torch.zeros(Sp, dtype=torch.bool, device=x.device)
        vm[:S] = valid_mask.reshape(-1)
    bits = _valid_bits(vm, Sp, x.device)
    w = ops.audio_pool_weights(a, Sp, block_size, bits, lambda_w)
    return ops.pool_chunks(xh, Sp, block_size, weights=w).view(B, H, Sp // block_size, D)


def compute_audio_spatial_concentration_gate(token_norms: torch.Tensor,
                                             valid_mask: Optional[torch.Tensor] = None,
                                             alpha: float = 5.0, beta: float = 2.0) -> torch.Tensor:
    """g_a = sigmoid(alpha * CV - beta), CV = std / (mean + 1e-6) of the (valid)
    token norms (bsa_interface.py:866-899); a 0-dim fp32 device tensor."""
    a = token_norms.reshape(-1).float()
    if valid_mask is None:
        mean = a.mean()
        var = (a - mean).square().mean()
    else:
        m = valid_mask.reshape(-1).float()
        n = m.sum().clamp(min=1.0)
        mean = (a * m).sum() / n
        var = ((a - mean).square() * m).sum() / n
    return torch.sigmoid(alpha * (var.sqrt() / (mean + 1e-6)) - beta)


def compute_timestep_reliability_gate(timestep_ratio: torch.Tensor, mode: str = "power",
                                      power: float = 1.5, scale: float = 10.0,
                                      threshold: float = 0.7) -> torch.Tensor:
    """r_t = (1 - t)^power ("power") or sigmoid(scale * (threshold - t))
    (bsa_interface.py:831-863)."""
    t = torch.as_tensor(timestep_ratio)
    if mode == "power":
        return (1.0 - t.clamp(0.0, 1.0)) ** power
    return torch.sigmoid(scale * (threshold - t))


def make_guidance(chunk_k, *, variance_gamma: float = 0.0, audio_token_norms=None,
                  audio_gate=None, audio_gamma=None, audio_weighted_lambda: float = 0.0,
                  score_modifier=None, n_chunks_k: Optional[int] = None, device=None) -> Optional[dict]:
    """The guidance a plan carries (None when nothing modulates the selection).
    audio_token_norms: per key token on the keys' grid (THW order); audio_gate: the
    gate g (tensor or float, default 1); audio_gamma: gamma_a (tensor or float,
    default 0); score_modifier: an additive boost per key chunk ([N_k] or
    broadcastable [1, 1, 1, N_k])."""
    norms = None
    if audio_token_norms is not None and audio_token_norms.numel() > 0:
        norms = audio_token_norms.reshape(-1).to(device=device, dtype=torch.float32).contiguous()
    gamma_a = 0.0 if audio_gamma is None else float(audio_gamma)
    has_audio = norms is not None and gamma_a > 0
    path_b = norms is not None and audio_weighted_lambda > 0
    gate = None
    if has_audio and audio_gate is not None:
        gate = torch.as_tensor(audio_gate, device=device).reshape(-1)[:1].to(torch.float32).contiguous()
    mod = None
    if score_modifier is not None:
        mod = torch.as_tensor(score_modifier, device=device).to(torch.float32).reshape(-1)
        if n_chunks_k is not None and mod.numel() == 1:
            mod = mod.expand(n_chunks_k)
        if n_chunks_k is not None and mod.numel() != n_chunks_k:
            raise NotImplementedError("score_modifier must be one value per key chunk")
        mod = mod.contiguous()
    if not (variance_gamma > 0 or has_audio or path_b or mod is not None):
        return None
    return dict(chunk_k=tuple(int(c) for c in chunk_k), variance_gamma=float(variance_gamma),
                norms=norms, audio=has_audio, gate=gate, audio_gamma=gamma_a,
                lambda_w=float(audio_weighted_lambda) if path_b else 0.0, modifier=mod)


def guidance_inputs(plan, g: dict, v_re: torch.Tensor):
    """(k_weights, col_scale) of a guided plan for its chunk-ordered V."""
    u = plan.uniform
    seq_k, ck = u["seq_k"], u["chunk_k"]
    bits = plan.tile_bits
    rho = sal = weights = None
    if g["variance_gamma"] > 0:
        if v_re is None:
            raise ValueError("variance guidance needs V")
        rho = ops.variance_density(v_re, seq_k, g["chunk_k"], bits)
    if g["norms"] is not None:
        a = ops.gather_values(g["norms"], plan.grid_k, plan.grid_padded_k, plan.src_idx_k)
        if g["audio"]:
            sal = ops.audio_saliency(a, seq_k, ck, bits)
        if g["lambda_w"] > 0:
            weights = ops.audio_pool_weights(a, seq_k, ck, bits, g["lambda_w"])
    scale = None
    if rho is not None or sal is not None or g["modifier"] is not None:
        scale = ops.guidance_scale(seq_k // ck, plan.tile_bits.device, rho=rho,
                                   variance_gamma=g["variance_gamma"], saliency=sal,
                                   audio_gate=g["gate"], audio_gamma=g["audio_gamma"],
                                   modifier=g["modifier"])
    return weights, scale


__all__ = ["compute_channel_variance_density", "compute_block_audio_saliency",
           "audio_weighted_mean_pooling_compression", "compute_audio_spatial_concentration_gate",
           "compute_timestep_reliability_gate", "make_guidance", "guidance_inputs"]
