"""Seeded synthetic inputs for the parity fixtures.

Generated with torch's CPU generator, so the same seeds give the same values on
any machine with the same torch build; the fixtures therefore store seeds and
reference outputs, not the input tensors.

Value models (benchmark configs):
* ``normal``: q, k, v ~ N(0, 1) (config 0).
* ``zoned``: each 8x8x8 macro-zone of the padded grid holds tokens
  ``zone_mean + 0.3 * noise`` with zone_mean, noise ~ N(0, 0.5^2) (configs 1-2),
  optionally times a per-zone amplitude U(lo, hi) so that zone densities differ.
* ``aniso``: zone_mean + sum over the axes d of w_d(zone) * wave_d(zone, position
  along d) + 0.1 * noise, with random per-zone axis weights, so zones are
  anisotropic and every candidate shape family (64- and 128-token) occurs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


@dataclass
class Case:
    name: str
    grid: Tuple[int, int, int]          # unpadded T, H, W
    heads: int
    head_dim: int
    values: str = "normal"              # "normal" | "zoned" | "aniso"
    amp: Optional[Tuple[float, float]] = None
    audio: bool = True
    audio_tokens: int = 32
    method: str = "ivpq"
    sparsity: Optional[float] = 0.75
    cdf_threshold: Optional[float] = 0.9
    lambda_a: float = 0.5
    tau_128: float = 0.15
    lambda_128: float = 1.0
    seed: int = 0
    extra: dict = field(default_factory=dict)
    # uniform fixed-shape path (flash_attn_bsa_3d) when set: q / key chunk shapes
    chunk_q: Optional[Tuple[int, int, int]] = None
    chunk_k: Optional[Tuple[int, int, int]] = None
    # guided uniform path (flash_attn_bsa_3d_variance_guided / _audio_guided) when set:
    # kind "variance" (variance_gamma) or "audio" (gate, audio_gamma, lambda_w,
    # variance_gamma)
    guidance: Optional[dict] = None
    # bias rectification of the uniform path (bsa_rectified_sparse_attn /
    # bsa_taylor_sparse_attn, bias_rectification.py:261-446) when set: kind
    # "rectified" or "taylor" (alpha_f), optional variance_gamma for a score modifier
    correction: Optional[dict] = None

    @property
    def uniform(self):
        return self.chunk_q is not None

    @property
    def grid_padded(self):
        if self.uniform:
            # the uniform dispatch pads each axis to the larger chunk extent
            # (wan_video_dit.py:473-481)
            m = [max(a, b) for a, b in zip(self.chunk_q, self.chunk_k)]
            return tuple(int(math.ceil(x / c) * c) for x, c in zip(self.grid, m))
        return tuple(int(math.ceil(x / 8) * 8) for x in self.grid)

    @property
    def needs_pad(self):
        return self.grid_padded != tuple(self.grid)


CASES = {
    # benchmark config 0: 4 heads, D=64, 4x8x8 grid (padded to 8x8x8), 32 audio tokens,
    # top-k 2 of 8 blocks (sparsity 0.75) + cumulative mass 0.9.
    "c0": Case("c0", (4, 8, 8), 4, 64),
    "c0_tau25_penalty": Case("c0_tau25_penalty", (4, 8, 8), 4, 64, method="penalty", tau_128=0.25),
    # anisotropic zones + penalty matching with a strong 128-token bonus: mixed 64/128 shapes
    "mixed_d64": Case("mixed_d64", (13, 14, 21), 2, 64, values="aniso", amp=(0.02, 1.0),
                      method="penalty", sparsity=0.9, cdf_threshold=0.5, tau_128=0.8,
                      lambda_128=3.0, seed=10),
    "mixed_d128_penalty": Case("mixed_d128_penalty", (5, 9, 16), 2, 128, values="aniso",
                               amp=(0.02, 1.0), method="penalty", sparsity=0.92,
                               cdf_threshold=0.9, tau_128=0.8, lambda_128=3.0, seed=33),
    "topk_only": Case("topk_only", (6, 11, 13), 2, 64, values="aniso", amp=(0.02, 1.0),
                      method="penalty", sparsity=0.8, cdf_threshold=None, tau_128=0.8,
                      lambda_128=3.0, seed=30),
    "cdf_only": Case("cdf_only", (6, 11, 13), 2, 64, values="aniso", amp=(0.02, 1.0),
                     method="penalty", sparsity=None, cdf_threshold=0.6, tau_128=0.8,
                     lambda_128=3.0, seed=40, audio=False),
    # IVPQ on anisotropic zones (64-token shapes of every orientation)
    "aniso_ivpq": Case("aniso_ivpq", (13, 14, 21), 2, 64, values="aniso", amp=(0.05, 1.0),
                       sparsity=0.9, cdf_threshold=0.5, tau_128=0.5, seed=10),
    "nopad_bf16": Case("nopad_bf16", (8, 8, 16), 2, 64, values="aniso", amp=(0.1, 1.0),
                       sparsity=0.75, cdf_threshold=0.9, seed=50),
}

# Uniform fixed-shape path (flash_attn_bsa_3d, bsa_interface.py:1123-1176).
UNIFORM_CASES = {
    # 4x4x4 chunks with the training configs' sparsity 0.75 / cdf 0.2; padded grid
    "u64_pad": Case("u64_pad", (6, 10, 12), 2, 64, values="aniso", amp=(0.05, 1.0), audio=False,
                    sparsity=0.75, cdf_threshold=0.2, chunk_q=(4, 4, 4), chunk_k=(4, 4, 4),
                    seed=60),
    # 4x4x8 chunks (the function's default), no padding, top-k only, head_dim 128
    "u128_nopad": Case("u128_nopad", (8, 8, 16), 2, 128, values="aniso", amp=(0.1, 1.0),
                       audio=False, sparsity=0.5, cdf_threshold=None, chunk_q=(4, 4, 8),
                       chunk_k=(4, 4, 8), seed=61),
    # 64-token q chunks against 128-token key chunks, cumulative mass only, padded
    "umix_cdf": Case("umix_cdf", (5, 9, 14), 2, 64, values="aniso", amp=(0.05, 1.0), audio=False,
                     sparsity=None, cdf_threshold=0.6, chunk_q=(4, 4, 4), chunk_k=(4, 4, 8),
                     seed=62),
    # three chunks (an odd number of tiles), head_dim 128, top-k + cumulative mass
    "u_odd_d128": Case("u_odd_d128", (3, 4, 12), 2, 128, audio=False, sparsity=0.5,
                       cdf_threshold=0.9, chunk_q=(4, 4, 4), chunk_k=(4, 4, 4), seed=63),
}

# Guided uniform path: per-key-chunk score scale from V's channel-variance density
# (flash_attn_bsa_3d_variance_guided, bsa_interface.py:1179-1260) and/or the audio
# saliency of the a2v norms, with optional audio-weighted key pooling
# (flash_attn_bsa_3d_audio_guided, :1395-1501).  Gate and gains are bf16-exact.
GUIDED_CASES = {
    # variance only, padded grid (masked statistics), 4x4x4 chunks, top-k + cdf
    "g_var_pad": Case("g_var_pad", (6, 10, 12), 2, 64, values="aniso", amp=(0.05, 1.0),
                      audio=False, sparsity=0.75, cdf_threshold=0.2, chunk_q=(4, 4, 4),
                      chunk_k=(4, 4, 4), seed=80, guidance=dict(kind="variance", variance_gamma=1.0)),
    # variance only, no padding, 4x4x8 chunks (4 frames of 32), head_dim 128, top-k only
    "g_var_d128": Case("g_var_d128", (8, 16, 24), 2, 128, values="aniso", amp=(0.1, 1.0),
                       audio=False, sparsity=0.5, cdf_threshold=None, chunk_q=(4, 4, 8),
                       chunk_k=(4, 4, 8), seed=81, guidance=dict(kind="variance", variance_gamma=2.0)),
    # audio saliency with the concentration gate and audio-weighted key pooling, padded
    "g_audio_pathb": Case("g_audio_pathb", (6, 10, 12), 2, 64, values="aniso", amp=(0.05, 1.0),
                          sparsity=0.75, cdf_threshold=0.5, chunk_q=(4, 4, 4), chunk_k=(4, 4, 4),
                          seed=82, guidance=dict(kind="audio", gate=0.625, audio_gamma=1.5,
                                                 lambda_w=1.0, variance_gamma=0.0)),
    # audio + variance in one boost bracket, cumulative mass only, no padding
    "g_audio_var": Case("g_audio_var", (8, 8, 16), 2, 64, values="aniso", amp=(0.1, 1.0),
                        sparsity=None, cdf_threshold=0.6, chunk_q=(4, 4, 8), chunk_k=(4, 4, 8),
                        seed=83, guidance=dict(kind="audio", gate=0.75, audio_gamma=1.0,
                                               lambda_w=0.0, variance_gamma=0.5)),
}
# Bias rectification (inference): the sparse output corrected for the mass of the
# chunks the selection dropped, on inputs already in the 3D-chunk order.
CORRECTION_CASES = {
    # Rectified SpaAttn on a padded grid, 4x4x4 chunks, top-k + cdf
    "r_rect_pad": Case("r_rect_pad", (6, 10, 12), 2, 64, values="aniso", amp=(0.05, 1.0),
                       audio=False, sparsity=0.75, cdf_threshold=0.5, chunk_q=(4, 4, 4),
                       chunk_k=(4, 4, 4), seed=90, correction=dict(kind="rectified")),
    # Rectified with a variance score modifier (selection on modified scores, A_pool on raw)
    "r_rect_mod": Case("r_rect_mod", (8, 12, 16), 2, 128, values="aniso", amp=(0.1, 1.0),
                       audio=False, sparsity=0.75, cdf_threshold=None, chunk_q=(4, 4, 4),
                       chunk_k=(4, 4, 4), seed=91,
                       correction=dict(kind="rectified", variance_gamma=1.0)),
    # Taylor (LIVEditor) merge on a padded grid, median split of the chunk variances
    "r_taylor_pad": Case("r_taylor_pad", (6, 10, 12), 2, 64, values="aniso", amp=(0.05, 1.0),
                         audio=False, sparsity=0.75, cdf_threshold=0.5, chunk_q=(4, 4, 4),
                         chunk_k=(4, 4, 4), seed=92, correction=dict(kind="taylor", alpha_f=0.5)),
    # Taylor with 128-token chunks, head_dim 128, no padding, cumulative mass only
    "r_taylor_d128": Case("r_taylor_d128", (8, 16, 16), 2, 128, values="aniso", amp=(0.1, 1.0),
                          audio=False, sparsity=None, cdf_threshold=0.6, chunk_q=(4, 4, 8),
                          chunk_k=(4, 4, 8), seed=93, correction=dict(kind="taylor", alpha_f=0.3)),
}
UNIFORM_CASES_ALL = dict(UNIFORM_CASES, **GUIDED_CASES, **CORRECTION_CASES)

ALL_CASES = dict(CASES, **UNIFORM_CASES_ALL)


@dataclass
class CrossCase:
    """Cross-modal BSA (flash_attn_bsa_cross, bsa_interface.py:1276-1392): each side
    is "3d" (shape = latent grid T, H, W) or "1d" (shape = (tokens,))."""
    name: str
    q_structure: str
    k_structure: str
    q_shape: Tuple[int, ...]
    k_shape: Tuple[int, ...]
    heads: int
    head_dim: int
    sparsity: Optional[float] = 0.75
    cdf_threshold: Optional[float] = None
    chunk_size_q: int = 64
    chunk_size_k: int = 64
    chunk_3d_q: Optional[Tuple[int, int, int]] = None
    chunk_3d_k: Optional[Tuple[int, int, int]] = None
    seed: int = 0

    @staticmethod
    def _len(shape):
        n = 1
        for x in shape:
            n *= x
        return n

    @property
    def Sq(self):
        return self._len(self.q_shape)

    @property
    def Sk(self):
        return self._len(self.k_shape)


CROSS_CASES = {
    # the v2a bridge's form: audio queries (1D, padded 150 -> 192) over video keys
    # (3D 6x10x12, padded to 8x12x12 with 4x4x4 chunks)
    "x_a2v": CrossCase("x_a2v", "1d", "3d", (150,), (6, 10, 12), 2, 64, sparsity=0.75,
                       cdf_threshold=0.5, chunk_3d_k=(4, 4, 4), seed=70),
    # video queries (3D 5x8x12 -> 8x8x12) over audio keys (1D 200 -> 256), head_dim 128
    "x_v2a": CrossCase("x_v2a", "3d", "1d", (5, 8, 12), (200,), 2, 128, sparsity=0.5,
                       cdf_threshold=None, chunk_3d_q=(4, 4, 4), seed=71),
    # two 3D grids of different sizes, 64- against 128-token chunks; neither side is
    # padded (the reference's bf16 pass cannot run with exactly one masked side: its
    # masked pooling is fp32, the unmasked one bf16, and cal_score rejects the mix)
    "x_3d3d": CrossCase("x_3d3d", "3d", "3d", (4, 8, 8), (8, 8, 16), 2, 64, sparsity=None,
                        cdf_threshold=0.6, chunk_3d_q=(4, 4, 4), chunk_3d_k=(4, 4, 8), seed=72),
}


def _side(gen, structure, shape, heads, D):
    """Seeded values of one side, [1, h, S, D] bf16 in its own token order."""
    if structure == "3d":
        T, H, W = shape
        Tg, Hg, Wg = (int(math.ceil(x / 8) * 8) for x in shape)
        x = _aniso(gen, heads, (Tg, Hg, Wg), D, (0.05, 1.0))
        x = x.reshape(heads, Tg, Hg, Wg, D)[:, :T, :H, :W].reshape(1, heads, T * H * W, D)
    else:
        (S,) = shape
        n_seg = int(math.ceil(S / 16))
        seg = torch.randn(heads, n_seg, 1, D, generator=gen) * 0.5
        x = (seg.expand(heads, n_seg, 16, D).reshape(heads, n_seg * 16, D)[:, :S]
             + 0.2 * torch.randn(heads, S, D, generator=gen)).reshape(1, heads, S, D)
    return x.to(torch.bfloat16)


def make_cross_inputs(case: CrossCase):
    """q, do [1, h, Sq, D]; k, v [1, h, Sk, D] bf16, unpadded, each in its own order."""
    out = {}
    for i, (name, st, shape) in enumerate((("q", case.q_structure, case.q_shape),
                                           ("k", case.k_structure, case.k_shape),
                                           ("v", case.k_structure, case.k_shape),
                                           ("do", case.q_structure, case.q_shape))):
        gen = torch.Generator().manual_seed(case.seed + i)
        out[name] = _side(gen, st, shape, case.heads, case.head_dim)
    return out


def _zoned(gen, heads, grid_p, D, amp):
    T, H, W = grid_p
    ZT, ZH, ZW = T // 8, H // 8, W // 8
    mean = torch.randn(heads, ZT, ZH, ZW, D, generator=gen) * 0.5
    noise = torch.randn(heads, T, H, W, D, generator=gen) * 0.5
    if amp is not None:
        a = torch.rand(ZT, ZH, ZW, generator=gen) * (amp[1] - amp[0]) + amp[0]
        mean = mean * a[None, :, :, :, None]
        scale = a.repeat_interleave(8, 0).repeat_interleave(8, 1).repeat_interleave(8, 2)
        noise = noise * scale[None, :, :, :, None]
    m = mean.repeat_interleave(8, 1).repeat_interleave(8, 2).repeat_interleave(8, 3)
    return (m + 0.3 * noise).reshape(heads, T * H * W, D)


def _aniso(gen, heads, grid_p, D, amp):
    T, H, W = grid_p
    ZT, ZH, ZW = T // 8, H // 8, W // 8
    mean = torch.randn(heads, ZT, 1, ZH, 1, ZW, 1, D, generator=gen) * 0.5
    wt = torch.randn(heads, ZT, 8, ZH, 1, ZW, 1, D, generator=gen) * 0.5
    wh = torch.randn(heads, ZT, 1, ZH, 8, ZW, 1, D, generator=gen) * 0.5
    ww = torch.randn(heads, ZT, 1, ZH, 1, ZW, 8, D, generator=gen) * 0.5
    w = torch.rand(3, ZT, 1, ZH, 1, ZW, 1, 1, generator=gen) ** 3
    w = w / w.sum(0, keepdim=True)
    x = mean + w[0] * wt + w[1] * wh + w[2] * ww
    noise = torch.randn(heads, ZT, 8, ZH, 8, ZW, 8, D, generator=gen) * 0.05
    if amp is not None:
        a = torch.rand(ZT, 1, ZH, 1, ZW, 1, 1, generator=gen) * (amp[1] - amp[0]) + amp[0]
        x = mean + a * (x - mean + noise)
    else:
        x = x + noise
    return x.reshape(heads, T * H * W, D)


def make_inputs(case: Case):
    """Returns dict of CPU tensors:
    q, k, v  [1, h, S_p, D] bf16, THW order, zero-padded (F.pad semantics);
    q_u, k_u, v_u [1, h, S, D] bf16 unpadded; do [1, h, S_p, D] bf16 (zero on padding);
    valid [S_p] bool or None; a2v [S, Da] bf16 or None; norms [S_p] bf16 or None."""
    T, H, W = case.grid
    Tp, Hp, Wp = case.grid_padded
    h, D = case.heads, case.head_dim
    out = {}
    # value models live on 8x8x8 macro-zones: generate on the grid rounded up to 8
    Tg, Hg, Wg = (int(math.ceil(x / 8) * 8) for x in (Tp, Hp, Wp))
    for i, name in enumerate(("q", "k", "v", "do")):
        gen = torch.Generator().manual_seed(case.seed + i)
        if case.values in ("zoned", "aniso") and name != "do":
            fn = _zoned if case.values == "zoned" else _aniso
            full = fn(gen, h, (Tg, Hg, Wg), D, case.amp)
            x = full.reshape(h, Tg, Hg, Wg, D)[:, :T, :H, :W].reshape(1, h, T * H * W, D)
        else:
            x = torch.randn(1, h, T * H * W, D, generator=gen)
        out[name + "_u"] = x.to(torch.bfloat16)
    for name in ("q", "k", "v", "do"):
        x = out[name + "_u"].view(1, h, T, H, W, D)
        xp = F.pad(x, (0, 0, 0, Wp - W, 0, Hp - H, 0, Tp - T))
        out[name] = xp.reshape(1, h, Tp * Hp * Wp, D).contiguous()
    if case.needs_pad:
        it = torch.arange(Tp)[:, None, None] < T
        ih = torch.arange(Hp)[None, :, None] < H
        iw = torch.arange(Wp)[None, None, :] < W
        out["valid"] = (it & ih & iw).reshape(-1).contiguous()
    else:
        out["valid"] = None
    if case.audio:
        gen = torch.Generator().manual_seed(case.seed + 4)
        a2v = torch.randn(T * H * W, case.audio_tokens * 2, generator=gen)
        gen = torch.Generator().manual_seed(case.seed + 5)
        # per-zone amplitude U(0.2, 2) on the cross-attention output (8x8x8 zones; a
        # grid padded only to a smaller chunk has a partial last zone)
        zt, zh, zw = (int(math.ceil(x / 8)) for x in (Tp, Hp, Wp))
        zscale = torch.rand(zt * zh * zw, generator=gen) * 1.8 + 0.2
        tt = torch.arange(T)[:, None, None] // 8
        hh = torch.arange(H)[None, :, None] // 8
        ww = torch.arange(W)[None, None, :] // 8
        zid = ((tt * zh + hh) * zw + ww).reshape(-1)
        a2v = (a2v * zscale[zid][:, None]).to(torch.bfloat16)
        out["a2v"] = a2v
        norms = a2v.norm(dim=-1)  # wan_video_dit.py:744, bf16 in -> bf16 out
        n3 = norms.reshape(T, H, W)
        out["norms_u"] = norms
        out["norms"] = F.pad(n3, (0, Wp - W, 0, Hp - H, 0, Tp - T)).reshape(-1).contiguous()
    else:
        out["a2v"] = None
        out["norms_u"] = None
        out["norms"] = None
    return out


# Producer side (RMSNorm + 3D RoPE, wan_video_dit.py:699-705): (grid, heads, head_dim, seed)
PRODUCER_CASES = {"p_rope_d128": ((3, 5, 7), 4, 128, 100), "p_rope_h1": ((2, 4, 6), 1, 128, 101)}


def make_producer_inputs(grid, heads, D, seed):
    """x [1, S, heads*D] bf16 (N(0, 4)) and gamma [heads*D] bf16 (1 + N(0, 1/16))."""
    f, h, w = grid
    S, C = f * h * w, heads * D
    gen = torch.Generator().manual_seed(seed)
    x = (torch.randn(1, S, C, generator=gen) * 2.0).to(torch.bfloat16)
    gamma = (1.0 + 0.25 * torch.randn(C, generator=gen)).to(torch.bfloat16)
    return x, gamma
