"""CPU oracle for Prism's dynamic block-sparse attention path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or the timed CPU baseline.  The product
(``prism_b200``) never imports it.

Two parts:

* ``libprism_oracle.so`` (``prism_oracle.c``): bit-exact restatement of the
  integer / selection side (zone statistics, shape choice, permutation,
  pooled-block scoring and hybrid top-k + cumulative-mass selection).
* numpy float64 block-sparse attention forward/backward, restating the Triton
  kernels ``_attn_fwd_bsa_varlen_align`` (flash_attn_bsa_varlen_mask.py:193-319),
  ``_attn_bwd_preprocess`` (common.py:94-111), ``_attn_bwd_dkdv_bsa_varlen_wrapper``
  (flash_attn_bsa_varlen_mask.py:564-704) and ``_attn_bwd_dq_bsa_varlen_align_wrapper``
  (:881-1014) as dense masked softmax attention over the selected 64-token tiles.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libprism_oracle.so")
_lib = None

SHAPES = [
    (4, 4, 4), (8, 2, 4), (8, 4, 2), (2, 4, 8), (2, 8, 4), (4, 2, 8), (4, 8, 2),
    (2, 8, 8), (8, 2, 8), (8, 8, 2), (4, 4, 8), (4, 8, 4), (8, 4, 4),
]  # dynamic_block_shape.py:6-23


def build() -> str:
    """Compile prism_oracle.c with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "prism_oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i64, i32, f32, f64 = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_double
        L.oracle_det_expf.argtypes = [f32]
        L.oracle_det_expf.restype = f32
        L.oracle_det_log2f.argtypes = [f32]
        L.oracle_det_log2f.restype = f32
        L.oracle_token_norms.argtypes = [P, i64, i32, P]
        L.oracle_zone_stats.argtypes = [P, i32, i32, i32, i32, i32, P, P, P, P, P]
        L.oracle_shape_select.argtypes = [P, P, P, i32, i32, i32, i32, f32, f32, f32, P, P, P]
        L.oracle_layout.argtypes = [P, i32, i32, i32, P, P, P, P]
        L.oracle_layout.restype = i64
        L.oracle_block_select.argtypes = [P, P, i32, i64, i32, P, i64, P, i32, f64, f64, P, P, P]
        L.oracle_block_select_uniform.argtypes = [P, P, i32, i64, i64, i32, i64, i64, i32, i32, P,
                                                  P, P, P, i32, f64, f64, P, P, P]
        L.oracle_variance_density.argtypes = [P, i32, i64, i32, i64, i32, i32, i32, P, P]
        L.oracle_audio_saliency.argtypes = [P, i64, i32, P, P]
        L.oracle_audio_pool_weights.argtypes = [P, i64, i32, P, f32, P]
        L.oracle_guidance_scale.argtypes = [i64, P, f32, P, f32, f32, P, P]
        L.oracle_uniform_pooled.argtypes = [P, P, i32, i64, i64, i32, i64, i64, i32, i32, P, P, P,
                                            P, P]
        L.oracle_correction_stats.argtypes = [P, i32, i32, i32, P, P, f32, P, P, P, P]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------ selection side
def token_norms(x_bits: np.ndarray) -> np.ndarray:
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    n, dim = x_bits.shape
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_token_norms(_p(x_bits), n, dim, _p(out))
    return out


def zone_stats(v_bits, grid, valid=None, norms_bits=None):
    """v_bits [heads, S, D] uint16 (bf16 bits).  Returns packed, axis_valid, audio."""
    v_bits = np.ascontiguousarray(v_bits, dtype=np.uint16)
    heads, S, D = v_bits.shape
    T, H, W = grid
    Nz = (T // 8) * (H // 8) * (W // 8)
    packed = np.empty((Nz, 25 * D), np.float32)
    axis_valid = np.empty((Nz, 24), np.uint8)
    audio = np.empty((Nz, 25), np.float32)
    valid = None if valid is None else np.ascontiguousarray(valid, dtype=np.uint8)
    norms_bits = None if norms_bits is None else np.ascontiguousarray(norms_bits, dtype=np.uint16)
    lib().oracle_zone_stats(_p(v_bits), heads, T, H, W, D, _p(valid), _p(norms_bits),
                            _p(packed), _p(axis_valid), _p(audio))
    return packed, axis_valid, audio


def shape_select(packed, axis_valid, audio, has_audio, method="ivpq", lambda_a=0.5,
                 tau_128=0.15, lambda_128=1.0):
    packed = np.ascontiguousarray(packed, np.float32)
    axis_valid = np.ascontiguousarray(axis_valid, np.uint8)
    audio = np.ascontiguousarray(audio, np.float32)
    Nz = packed.shape[0]
    D = packed.shape[1] // 25
    ids = np.empty(Nz, np.int64)
    g = np.empty((Nz, 3), np.float32)
    rho = np.empty(Nz, np.float32)
    m = {"ivpq": 0, "penalty": 1}[method]
    lib().oracle_shape_select(_p(packed), _p(axis_valid), _p(audio), int(bool(has_audio)), Nz, D,
                              m, lambda_a, tau_128, lambda_128, _p(ids), _p(g), _p(rho))
    return ids, g, rho


def layout(shape_ids, grid):
    shape_ids = np.ascontiguousarray(shape_ids, np.int64)
    T, H, W = grid
    S = T * H * W
    Nz = shape_ids.shape[0]
    src = np.empty(S, np.int64)
    inv = np.empty(S, np.int64)
    bot = np.empty(Nz * 8, np.int64)
    bt = np.empty((Nz * 8 + 1) * 2, np.int64)
    nb = lib().oracle_layout(_p(shape_ids), T, H, W, _p(src), _p(inv), _p(bot), _p(bt))
    return src, inv, bot, bt[: (nb + 1) * 2].reshape(nb + 1, 2), int(nb)


def selection_mode(sparsity, cdf_threshold):
    if sparsity is not None and cdf_threshold is not None:
        return 0
    if sparsity is None and cdf_threshold is not None:
        return 1
    if sparsity is not None and cdf_threshold is None:
        return 2
    raise ValueError("Either sparsity or cdf_threshold must be provided")


def block_select(q_re_bits, k_re_bits, valid_re, block_tiles, nb, sparsity, cdf_threshold,
                 want_blocks=False):
    """Returns (bits_q [h, N_tiles, WQ] u32, bits_k [h, N_tiles, WQ] u32, sel_blocks or None)."""
    q_re_bits = np.ascontiguousarray(q_re_bits, np.uint16)
    k_re_bits = np.ascontiguousarray(k_re_bits, np.uint16)
    heads, S, D = q_re_bits.shape
    n_tiles = S // 64
    wq = (n_tiles + 31) // 32
    bits_q = np.zeros((heads, n_tiles, wq), np.uint32)
    bits_k = np.zeros((heads, n_tiles, wq), np.uint32)
    sel = np.zeros((heads, nb, nb), np.uint8) if want_blocks else None
    valid_re = None if valid_re is None else np.ascontiguousarray(valid_re, np.uint8)
    bt = np.ascontiguousarray(block_tiles, np.int64)
    mode = selection_mode(sparsity, cdf_threshold)
    lib().oracle_block_select(_p(q_re_bits), _p(k_re_bits), heads, S, D, _p(valid_re), nb, _p(bt),
                              mode, float(sparsity if sparsity is not None else 0.0),
                              float(cdf_threshold if cdf_threshold is not None else 0.0),
                              _p(bits_q), _p(bits_k), _p(sel))
    return bits_q, bits_k, sel


def uniform_layout(grid_padded, chunk, n_rows=None):
    """3D-chunk order of the uniform path (rearrange_THW_to_3d_block,
    bsa_interface.py:1105-1109): src_idx [n_rows] (padded THW index of each
    row; rows past the grid hold the sentinel Tp*Hp*Wp) and inv_idx [Tp*Hp*Wp]."""
    Tp, Hp, Wp = grid_padded
    ct, ch, cw = chunk
    S = Tp * Hp * Wp
    n_rows = S if n_rows is None else n_rows
    order = np.arange(S).reshape(Tp // ct, ct, Hp // ch, ch, Wp // cw, cw)
    order = order.transpose(0, 2, 4, 1, 3, 5).reshape(-1)
    src = np.full(n_rows, S, np.int64)
    src[:S] = order
    inv = np.empty(S, np.int64)
    inv[order] = np.arange(S)
    return src, inv


def block_select_uniform(q_re_bits, k_re_bits, seq_q, seq_k, chunk_q, chunk_k, q_valid, k_valid,
                         sparsity, cdf_threshold, want_chunks=False, k_weights=None,
                         col_scale=None):
    """Uniform-path selection (oracle_block_select_uniform).  q_re_bits [h, Sq, D]
    in the q chunk order, k_re_bits [h, Sk, D] in the key chunk order (bf16 bits);
    q_valid [Sq] / k_valid [Sk]: rows the q / k pooling counts and key validity
    (None = every row).  Guided selection: k_weights [seq_k] f32 (Path B key
    pooling weights) and col_scale [nk] f32 (per-key-chunk score scale).
    Returns (bits_q [h, Sq/64, ceil(Sk/2048)], bits_k [h, Sk/64, ceil(Sq/2048)],
    sel_chunks [h, nq, nk] or None)."""
    q_re_bits = np.ascontiguousarray(q_re_bits, np.uint16)
    k_re_bits = np.ascontiguousarray(k_re_bits, np.uint16)
    heads, Sq, D = q_re_bits.shape
    Sk = k_re_bits.shape[1]
    nqt, nkt = Sq // 64, Sk // 64
    bits_q = np.zeros((heads, nqt, (nkt + 31) // 32), np.uint32)
    bits_k = np.zeros((heads, nkt, (nqt + 31) // 32), np.uint32)
    sel = (np.zeros((heads, seq_q // chunk_q, seq_k // chunk_k), np.uint8) if want_chunks else None)
    q_valid = None if q_valid is None else np.ascontiguousarray(q_valid, np.uint8)
    k_valid = None if k_valid is None else np.ascontiguousarray(k_valid, np.uint8)
    k_weights = None if k_weights is None else np.ascontiguousarray(k_weights, np.float32)
    col_scale = None if col_scale is None else np.ascontiguousarray(col_scale, np.float32)
    mode = selection_mode(sparsity, cdf_threshold)
    lib().oracle_block_select_uniform(
        _p(q_re_bits), _p(k_re_bits), heads, Sq, Sk, D, seq_q, seq_k, chunk_q, chunk_k,
        _p(q_valid), _p(k_valid), _p(k_weights), _p(col_scale), mode,
        float(sparsity if sparsity is not None else 0.0),
        float(cdf_threshold if cdf_threshold is not None else 0.0), _p(bits_q), _p(bits_k),
        _p(sel))
    return bits_q, bits_k, sel


# ------------------------------------------------------------ guided selection
def variance_density(v_re_bits, seq_k, chunk, k_valid):
    """oracle_variance_density: rho [seq_k / chunk volume] f32 of chunk-ordered V
    [h, Sk, D] (bf16 bits); chunk = (ct, ch, cw); k_valid [Sk] or None."""
    v = np.ascontiguousarray(v_re_bits, np.uint16)
    heads, Sk, D = v.shape
    ct, ch, cw = (int(c) for c in chunk)
    rho = np.zeros(seq_k // (ct * ch * cw), np.float32)
    kv = None if k_valid is None else np.ascontiguousarray(k_valid, np.uint8)
    lib().oracle_variance_density(_p(v), heads, Sk, D, seq_k, ct, ch, cw, _p(kv), _p(rho))
    return rho


def audio_saliency(norms_re, seq_k, chunk, k_valid):
    """oracle_audio_saliency: masked chunk means of the norms / their max."""
    x = np.ascontiguousarray(norms_re, np.float32)
    out = np.zeros(seq_k // chunk, np.float32)
    kv = None if k_valid is None else np.ascontiguousarray(k_valid, np.uint8)
    lib().oracle_audio_saliency(_p(x), seq_k, chunk, _p(kv), _p(out))
    return out


def audio_pool_weights(norms_re, seq_k, chunk, k_valid, lambda_w):
    """oracle_audio_pool_weights: Path B per-row key pooling weights [seq_k] f32."""
    x = np.ascontiguousarray(norms_re, np.float32)
    out = np.zeros(seq_k, np.float32)
    kv = None if k_valid is None else np.ascontiguousarray(k_valid, np.uint8)
    lib().oracle_audio_pool_weights(_p(x), seq_k, chunk, _p(kv), float(lambda_w), _p(out))
    return out


def guidance_scale(n, rho=None, variance_gamma=0.0, saliency=None, gate=1.0, audio_gamma=0.0,
                   modifier=None):
    """oracle_guidance_scale: 1 + boost per key chunk."""
    f = lambda a: None if a is None else np.ascontiguousarray(a, np.float32)
    rho, saliency, modifier = f(rho), f(saliency), f(modifier)
    out = np.zeros(n, np.float32)
    lib().oracle_guidance_scale(n, _p(rho), float(variance_gamma), _p(saliency), float(gate),
                                float(audio_gamma), _p(modifier), _p(out))
    return out


# ---------------------------------------------------------- bias rectification
def uniform_pooled(q_re_bits, k_re_bits, seq_q, seq_k, chunk_q, chunk_k, q_valid, k_valid):
    """oracle_uniform_pooled: (qc [h, nq, D], kc [h, nk, D], raw scores [h, nq, nk]) f32."""
    q = np.ascontiguousarray(q_re_bits, np.uint16)
    k = np.ascontiguousarray(k_re_bits, np.uint16)
    heads, Sq, D = q.shape
    Sk = k.shape[1]
    nq, nk = seq_q // chunk_q, seq_k // chunk_k
    qc = np.zeros((heads, nq, D), np.float32)
    kc = np.zeros((heads, nk, D), np.float32)
    sc = np.zeros((heads, nq, nk), np.float32)
    qv = None if q_valid is None else np.ascontiguousarray(q_valid, np.uint8)
    kv = None if k_valid is None else np.ascontiguousarray(k_valid, np.uint8)
    lib().oracle_uniform_pooled(_p(q), _p(k), heads, Sq, Sk, D, seq_q, seq_k, chunk_q, chunk_k,
                                _p(qv), _p(kv), _p(qc), _p(kc), _p(sc))
    return qc, kc, sc


def correction_stats(scores, sel, chunk_valid, sm_scale, want_a_rect=False):
    """oracle_correction_stats: (R [h, nq], M [h, nq], nonsel [h, nq, ceil(nk/64)] u64,
    a_rect [h, nq, nk] or None) from raw scores, the chunk selection and validity."""
    sc = np.ascontiguousarray(scores, np.float32)
    heads, nq, nk = sc.shape
    sl = np.ascontiguousarray(sel, np.uint8)
    cv = np.ascontiguousarray(chunk_valid, np.uint8)
    R = np.zeros((heads, nq), np.float32)
    M = np.zeros((heads, nq), np.float32)
    nonsel = np.zeros((heads, nq, (nk + 63) // 64), np.uint64)
    a_rect = np.zeros((heads, nq, nk), np.float32) if want_a_rect else None
    lib().oracle_correction_stats(_p(sc), heads, nq, nk, _p(sl), _p(cv), float(sm_scale), _p(R),
                                  _p(M), _p(nonsel), _p(a_rect))
    return R, M, nonsel, a_rect


def rectified_output(o_spa, R, a_rect, v_cmp, chunk_q):
    """O' = R_n O_spa + (A_pool * unselected) V_cmp per q chunk, float64
    (_rectified_correction_pytorch, bias_rectification.py:335-377).  o_spa [h, S, D]."""
    h, S, D = o_spa.shape
    o_ncri = np.einsum("hab,hbd->had", a_rect.astype(np.float64), v_cmp.astype(np.float64))
    return (np.repeat(R.astype(np.float64), chunk_q, axis=1)[:, :, None] * o_spa
            + np.repeat(o_ncri, chunk_q, axis=1))


def taylor_output(q, o_spa, lse_spa, k_cmp, v_cmp, nonsel_dense, flat, log_counts, chunk_q,
                  sm_scale):
    """_taylor_merge_pytorch (bias_rectification.py:190-257) in float64: for flat q
    chunks, softmax over the unselected pooled keys of q k_cmp * sm_scale + log
    count, merged with the sparse output by log-sum-exp.  q, o_spa [h, S, D],
    lse_spa [h, S] (natural log), k_cmp / v_cmp [h, nk, D], nonsel_dense
    [h, nq, nk] bool, flat [h, nq] bool, log_counts [nk]."""
    q = q.astype(np.float64)
    out = o_spa.astype(np.float64).copy()
    h, S, D = q.shape
    for hh in range(h):
        for a in np.nonzero(flat[hh])[0]:
            rows = slice(a * chunk_q, (a + 1) * chunk_q)
            m = nonsel_dense[hh, a]
            if not m.any():
                continue
            z = q[hh, rows] @ k_cmp[hh, m].astype(np.float64).T * sm_scale + log_counts[m][None]
            zm = z.max(axis=1, keepdims=True)
            p = np.exp(z - zm)
            l = p.sum(axis=1, keepdims=True)
            lse_t = (zm + np.log(l))[:, 0]
            o_t = (p / l) @ v_cmp[hh, m].astype(np.float64)
            ls = lse_spa[hh, rows].astype(np.float64)
            lm = np.maximum(ls, lse_t)
            tot = lm + np.log(np.exp(ls - lm) + np.exp(lse_t - lm))
            out[hh, rows] = (np.exp(ls - tot)[:, None] * out[hh, rows]
                             + np.exp(lse_t - tot)[:, None] * o_t)
    return out


# ---------------------------------------------------------------- producer side
def f32_to_bf16_bits(x):
    """float32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def rms_norm(x_bits, gamma, eps=1e-6):
    """torch.nn.RMSNorm of bf16 rows [S, C] (x * rsqrt(mean(x^2) + eps)) * gamma in
    float32 (mean in float64 here), rounded to bf16 bits."""
    x = bf16_bits_to_f32(x_bits)
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    r = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
    y = (x * r).astype(np.float32) * np.asarray(gamma, np.float32)
    return f32_to_bf16_bits(y.astype(np.float32))


def rope_apply(y_bits, rope_cs, D):
    """rope_apply_head_dim (wan_video_dit.py:177-182) of bf16 rows [S, H*D]: each
    (even, odd) pair times cos + i sin in float64, the result rounded to float32,
    then to bf16 (torch's double -> bf16 conversion).  rope_cs [S, D/2, 2]."""
    y = bf16_bits_to_f32(y_bits).astype(np.float64)
    S, C = y.shape
    H = C // D
    p = y.reshape(S, H, D // 2, 2)
    c = rope_cs[:, None, :, 0]
    s = rope_cs[:, None, :, 1]
    re = p[..., 0] * c - p[..., 1] * s
    im = p[..., 0] * s + p[..., 1] * c
    out = np.stack([re, im], axis=-1).reshape(S, C).astype(np.float32)
    return f32_to_bf16_bits(out)


def bits_to_dense(bits: np.ndarray, n_cols: int) -> np.ndarray:
    """[..., rows, WQ] u32 -> [..., rows, n_cols] bool."""
    b = bits.view(np.uint8).reshape(*bits.shape[:-1], bits.shape[-1] * 4)
    d = np.unpackbits(b, axis=-1, bitorder="little").astype(bool)
    return d[..., :n_cols]


def dense_to_bits(dense: np.ndarray) -> np.ndarray:
    n_cols = dense.shape[-1]
    wq = (n_cols + 31) // 32
    pad = np.zeros((*dense.shape[:-1], wq * 32), bool)
    pad[..., :n_cols] = dense
    return np.packbits(pad, axis=-1, bitorder="little").view(np.uint32)


def tile_lists_to_dense(tile_block_indices, lens, n_tiles):
    """Reference selection (tile_block_indices [B,h,Nt,W], lens [B,h,Nt]) -> [h, Nt, Nt] bool."""
    tbi = np.asarray(tile_block_indices)[0]
    ln = np.asarray(lens)[0]
    h, nt, w = tbi.shape
    dense = np.zeros((h, nt, n_tiles), bool)
    pos = np.arange(w)[None, None, :]
    keep = pos < ln[..., None]
    hh, rr, cc = np.nonzero(keep)
    dense[hh, rr, tbi[hh, rr, cc]] = True
    return dense


# ------------------------------------------------------------ attention side
def token_mask(bits_q: np.ndarray, valid_re, S: int, Sk: int = None) -> np.ndarray:
    """[h, S, Sk] bool: query token i may attend key token j (Sk defaults to S)."""
    Sk = S if Sk is None else Sk
    dense = bits_to_dense(bits_q, Sk // 64)[:, :S // 64]  # [h, Nq, Nk]
    m = np.repeat(np.repeat(dense, 64, axis=1), 64, axis=2)
    if valid_re is not None:
        m = m & np.asarray(valid_re, bool)[None, None, :]
    return m


_ROW_BLOCK = 512  # query rows per dense block (keeps the temporaries small)


def _block_mask(dense_h, valid, r0, r1, Sk):
    """[r1 - r0, Sk] token mask of query rows [r0, r1) from one head's tile mask."""
    t = dense_h[r0 // 64:(r1 + 63) // 64]                      # [tiles, Nk]
    m = np.repeat(np.repeat(t, 64, axis=0)[r0 % 64:r0 % 64 + (r1 - r0)], 64, axis=1)[:, :Sk]
    if valid is not None:
        m = m & valid[None, :]
    return m


def _blocks(bits_q, valid_re, S, Sk):
    dense = bits_to_dense(bits_q, Sk // 64)[:, :S // 64]
    valid = None if valid_re is None else np.asarray(valid_re, bool)
    for hh in range(dense.shape[0]):
        for r0 in range(0, S, _ROW_BLOCK):
            r1 = min(S, r0 + _ROW_BLOCK)
            yield hh, r0, r1, _block_mask(dense[hh], valid, r0, r1, Sk)


def bsa_forward(q, k, v, bits_q, valid_re, sm_scale=None):
    """Float64 restatement of the sparse forward.  q [h, S, D], k, v [h, Sk, D] float.

    Returns (o [h,S,D], lse [h,S]) with lse natural-log (bsa_interface.py:382-383);
    rows with no selected valid key give o = 0 and lse = -inf, as the
    reference's l_i = 1 initialisation does (flash_attn_bsa_varlen_mask.py:264).
    Dense masked softmax per head over blocks of query rows."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    h, S, D = q.shape
    Sk = k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    o = np.zeros((h, S, D))
    lse = np.zeros((h, S))
    for hh, r0, r1, m in _blocks(bits_q, valid_re, S, Sk):
        s = np.where(m, (q[hh, r0:r1] @ k[hh].T) * sm_scale, -np.inf)
        mx = s.max(-1, keepdims=True)
        empty = ~np.isfinite(mx)
        mx = np.where(empty, 0.0, mx)
        p = np.exp(s - mx)
        l = p.sum(-1, keepdims=True)
        lsafe = np.where(l > 0, l, 1.0)
        o[hh, r0:r1] = (p / lsafe) @ v[hh]
        lse[hh, r0:r1] = np.where(empty[:, 0], -np.inf, (mx + np.log(lsafe))[:, 0])
    return o, lse


def bsa_backward(q, k, v, o, do, bits_q, valid_re, sm_scale=None):
    """Float64 gradient of bsa_forward given the (possibly rounded) output o.

    Delta = rowsum(o * do) uses the stored output, as _attn_bwd_preprocess does."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    o = np.asarray(o, np.float64)
    do = np.asarray(do, np.float64)
    h, S, D = q.shape
    Sk = k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    dq = np.zeros((h, S, D))
    dk = np.zeros((h, Sk, D))
    dv = np.zeros((h, Sk, D))
    for hh, r0, r1, m in _blocks(bits_q, valid_re, S, Sk):
        s = np.where(m, (q[hh, r0:r1] @ k[hh].T) * sm_scale, -np.inf)
        mx = s.max(-1, keepdims=True)
        mx = np.where(np.isfinite(mx), mx, 0.0)
        p = np.exp(s - mx)
        l = p.sum(-1, keepdims=True)
        p = p / np.where(l > 0, l, 1.0)
        delta = (o[hh, r0:r1] * do[hh, r0:r1]).sum(-1, keepdims=True)
        dp = do[hh, r0:r1] @ v[hh].T
        ds = p * (dp - delta)
        dq[hh, r0:r1] = (ds @ k[hh]) * sm_scale
        dk[hh] += (ds.T @ q[hh, r0:r1]) * sm_scale
        dv[hh] += p.T @ do[hh, r0:r1]
    return dq, dk, dv


# -------------------------------------------------------------- full path
def dynamic_forward_selection(q_bits, k_bits, v_bits, grid, *, method, sparsity, cdf_threshold,
                              norms_bits=None, valid=None, lambda_a=0.5, tau_128=0.15,
                              lambda_128=1.0, shape_ids=None):
    """Oracle for steps (1)-(5) of flash_attn_bsa_3d_dynamic
    (dynamic_block_attention.py:233-319).  Inputs are bf16 bit arrays [h,S,D].

    Returns a dict with shape_ids, src_idx, inv_idx, block_tiles, nb, valid_re,
    q_re/k_re/v_re (bits), bits_q, bits_k."""
    T, H, W = grid
    if shape_ids is None:
        packed, av, audio = zone_stats(v_bits, grid, valid, norms_bits)
        shape_ids, g, rho = shape_select(packed, av, audio, norms_bits is not None, method,
                                         lambda_a, tau_128, lambda_128)
    src, inv, bot, bt, nb = layout(shape_ids, grid)
    q_re = np.ascontiguousarray(q_bits[:, src])
    k_re = np.ascontiguousarray(k_bits[:, src])
    v_re = np.ascontiguousarray(v_bits[:, src])
    valid_re = None if valid is None else np.ascontiguousarray(np.asarray(valid, np.uint8)[src])
    bq, bk, _ = block_select(q_re, k_re, valid_re, bt, nb, sparsity, cdf_threshold)
    return dict(shape_ids=np.asarray(shape_ids, np.int64), src_idx=src, inv_idx=inv,
                block_of_tile=bot, block_tiles=bt, nb=nb, valid_re=valid_re, q_re=q_re,
                k_re=k_re, v_re=v_re, bits_q=bq, bits_k=bk)
