"""Torch-facing wrappers of the C ABI (include/prism_bsa.h).

Every function takes CUDA tensors, allocates its outputs and workspaces with
torch's caching allocator, and enqueues the kernels on the current stream.
Nothing here computes on the CPU; a missing library or a non-CUDA tensor is an
error.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib

SELECT_MODES = {"topk_cdf": 0, "cdf": 1, "topk": 2}


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise _lib.PrismError("prism_b200 ops require CUDA tensors (no CPU fallback)")


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def padded_grid(grid: Tuple[int, int, int]) -> Tuple[int, int, int]:
    return tuple(int(math.ceil(int(x) / 8) * 8) for x in grid)


def selection_mode(sparsity, cdf_threshold) -> int:
    if sparsity is not None and cdf_threshold is None:
        return SELECT_MODES["topk"]
    if sparsity is None and cdf_threshold is not None:
        return SELECT_MODES["cdf"]
    if sparsity is not None and cdf_threshold is not None:
        return SELECT_MODES["topk_cdf"]
    raise ValueError("Either sparsity or cdf_threshold must be provided")


# ------------------------------------------------------------------- a2
def token_norms(x: torch.Tensor) -> torch.Tensor:
    """||x||_2 over the last dim, bf16 in/out (wan_video_dit.py:742-744)."""
    _check_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("token_norms expects bf16")
    xc = x.contiguous()
    dim = xc.shape[-1]
    n = xc.numel() // dim
    out = torch.empty(xc.shape[:-1], dtype=torch.bfloat16, device=x.device)
    _lib.call("prism_token_norms", _p(xc), n, dim, _p(out), _stream(x))
    return out


# --------------------------------------------------------------- a4-a7
def zone_stats(v_hsd: torch.Tensor, grid, grid_padded, valid: Optional[torch.Tensor] = None,
               norms: Optional[torch.Tensor] = None):
    """v_hsd: [heads, T*H*W, D] bf16 view (D contiguous) on the source grid.
    Returns packed [Nz, 25*D] f32, axis_valid [Nz, 24] u8, audio [Nz, 25] f32."""
    _check_cuda(v_hsd, valid, norms)
    heads, S, D = v_hsd.shape
    T, H, W = grid
    Tp, Hp, Wp = grid_padded
    if S != T * H * W:
        raise ValueError(f"sequence {S} != grid {grid}")
    if v_hsd.stride(2) != 1:
        raise ValueError("v must be contiguous in the head dim")
    Nz = (Tp // 8) * (Hp // 8) * (Wp // 8)
    dev = v_hsd.device
    packed = torch.empty(Nz, 25 * D, dtype=torch.float32, device=dev)
    axis_valid = torch.empty(Nz, 24, dtype=torch.uint8, device=dev)
    audio = torch.empty(Nz, 25, dtype=torch.float32, device=dev)
    ws = _ws(_lib.query("prism_zone_stats_workspace_bytes", Tp, Hp, Wp, D), dev)
    vm = None if valid is None else valid.to(torch.uint8).contiguous()
    nm = None if norms is None else norms.to(torch.bfloat16).contiguous()
    _lib.call("prism_zone_stats", _p(v_hsd), heads, v_hsd.stride(0), v_hsd.stride(1), T, H, W,
              Tp, Hp, Wp, D, _p(vm), _p(nm), _p(ws), _p(packed), _p(axis_valid), _p(audio),
              _stream(v_hsd))
    return packed, axis_valid, audio


def shape_select(packed, axis_valid, audio, has_audio: bool, method: str, lambda_a=0.5,
                 tau_128=0.15, lambda_128=1.0, want_diag=False):
    if method not in ("ivpq", "penalty"):
        raise ValueError(f"unknown dynamic-block method: {method!r}")
    _check_cuda(packed)
    Nz = packed.shape[0]
    D = packed.shape[1] // 25
    dev = packed.device
    ids = torch.empty(Nz, dtype=torch.int64, device=dev)
    g = torch.empty(Nz, 3, dtype=torch.float32, device=dev) if want_diag else None
    rho = torch.empty(Nz, dtype=torch.float32, device=dev) if want_diag else None
    _lib.call("prism_shape_select", _p(packed), _p(axis_valid), _p(audio), int(bool(has_audio)),
              Nz, D, 0 if method == "ivpq" else 1, float(lambda_a), float(tau_128),
              float(lambda_128), _p(ids), _p(g), _p(rho), _stream(packed))
    if want_diag:
        return ids, g, rho
    return ids


# ---------------------------------------------------------------- a8/a9
def build_layout(shape_ids: torch.Tensor, grid_padded):
    _check_cuda(shape_ids)
    Tp, Hp, Wp = grid_padded
    S = Tp * Hp * Wp
    n_tiles = S // 64
    dev = shape_ids.device
    ids = shape_ids.to(torch.int64).contiguous()
    src = torch.empty(S, dtype=torch.int32, device=dev)
    inv = torch.empty(S, dtype=torch.int32, device=dev)
    bot = torch.empty(n_tiles, dtype=torch.int32, device=dev)
    bt = torch.empty(n_tiles + 1, 2, dtype=torch.int32, device=dev)
    nb = torch.empty(1, dtype=torch.int32, device=dev)
    _lib.call("prism_build_layout", _p(ids), Tp, Hp, Wp, _p(src), _p(inv), _p(bot), _p(bt), _p(nb),
              _stream(ids))
    return dict(src_idx=src, inv_idx=inv, block_of_tile=bot, block_tiles=bt, n_blocks=nb)


def tile_valid(src_idx, valid, grid, grid_padded):
    _check_cuda(src_idx, valid)
    T, H, W = grid
    Tp, Hp, Wp = grid_padded
    n_rows = src_idx.numel()
    n_tiles = n_rows // 64
    dev = src_idx.device
    bits = torch.empty(n_tiles, dtype=torch.int64, device=dev)
    cnt = torch.empty(n_tiles, dtype=torch.int32, device=dev)
    vm = None if valid is None else valid.to(torch.uint8).contiguous()
    _lib.call("prism_tile_valid", _p(src_idx), n_rows, _p(vm), T, H, W, Tp, Hp, Wp, _p(bits),
              _p(cnt), _stream(src_idx))
    return bits, cnt


# -------------------------------------------------------------- a10/a17
def gather_rows(x_hsd: torch.Tensor, grid, grid_padded, src_idx: torch.Tensor) -> torch.Tensor:
    """x_hsd [heads, T*H*W, D] (D contiguous) -> [heads, len(src_idx), D] tile order,
    zero rows for padded tokens."""
    _check_cuda(x_hsd, src_idx)
    heads, S, D = x_hsd.shape
    T, H, W = grid
    Tp, Hp, Wp = grid_padded
    if x_hsd.stride(2) != 1:
        raise ValueError("rows must be contiguous")
    n_rows = src_idx.numel()
    out = torch.empty(heads, n_rows, D, dtype=x_hsd.dtype, device=x_hsd.device)
    _lib.call("prism_gather_rows", _p(x_hsd), x_hsd.stride(0), x_hsd.stride(1), heads, D, T, H, W,
              Tp, Hp, Wp, _p(src_idx), n_rows, _p(out), out.stride(0), _stream(x_hsd))
    return out


def scatter_rows(x_re: torch.Tensor, grid, grid_padded, inv_idx: torch.Tensor,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[heads, S_p, D] tile order -> out [heads, T*H*W, D] (any head/token strides)."""
    _check_cuda(x_re, inv_idx)
    heads, Sp, D = x_re.shape
    T, H, W = grid
    Tp, Hp, Wp = grid_padded
    if out is None:
        out = torch.empty(heads, T * H * W, D, dtype=x_re.dtype, device=x_re.device)
    _lib.call("prism_scatter_rows", _p(x_re), x_re.stride(0), heads, D, T, H, W, Tp, Hp, Wp,
              _p(inv_idx), _p(out), out.stride(0), out.stride(1), _stream(x_re))
    return out


def copy_rows(src: torch.Tensor, src_strides, dst: torch.Tensor, dst_strides, n_blocks: int,
              n_rows: int, row_elems: int) -> None:
    """dst rows <- src rows: for block o and row r, row_elems elements from
    src.data_ptr() + o * src_strides[0] + r * src_strides[1] to the same position of dst
    (strides in elements of src.dtype; every offset a multiple of 16 bytes)."""
    _check_cuda(src, dst)
    es = src.element_size()
    _lib.call("prism_copy_rows", _p(src), src_strides[0] * es, src_strides[1] * es, _p(dst),
              dst_strides[0] * es, dst_strides[1] * es, int(n_blocks), int(n_rows), int(row_elems) * es,
              _stream(src))


# -------------------------------------------------------------- a11-a14
def block_select(q_re, k_re, layout, tile_bits, sparsity, cdf_threshold):
    _check_cuda(q_re, k_re)
    heads, S, D = q_re.shape
    mode = selection_mode(sparsity, cdf_threshold)
    n_tiles = S // 64
    wq = (n_tiles + 31) // 32
    dev = q_re.device
    bits_q = torch.empty(heads, n_tiles, wq, dtype=torch.int32, device=dev)
    bits_k = torch.empty(heads, n_tiles, wq, dtype=torch.int32, device=dev)
    ws = _ws(_lib.query("prism_block_select_workspace_bytes", heads, S, D), dev)
    _lib.call("prism_block_select", _p(q_re), _p(k_re), heads, S, D, _p(layout["block_tiles"]),
              _p(layout["n_blocks"]), _p(tile_bits), mode,
              float(sparsity if sparsity is not None else 0.0),
              float(cdf_threshold if cdf_threshold is not None else 0.0), _p(ws), _p(bits_q),
              _p(bits_k), _stream(q_re))
    return bits_q, bits_k


# ------------------------------------------------------- uniform chunks
def uniform_layout(grid_padded, chunk, n_rows: int, device):
    """src_idx [n_rows] / inv_idx [Tp*Hp*Wp] int32 of the 3D-chunk order
    (rearrange_THW_to_3d_block, bsa_interface.py:1105-1109)."""
    Tp, Hp, Wp = grid_padded
    ct, ch, cw = chunk
    src = torch.empty(n_rows, dtype=torch.int32, device=device)
    inv = torch.empty(Tp * Hp * Wp, dtype=torch.int32, device=device)
    _lib.call("prism_uniform_layout", Tp, Hp, Wp, ct, ch, cw, n_rows, _p(src), _p(inv),
              ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    return src, inv


def block_select_uniform(q_re, k_re, seq_q: int, seq_k: int, chunk_q: int, chunk_k: int, q_bits,
                         k_bits, sparsity, cdf_threshold, k_weights=None, col_scale=None,
                         want_pooled: bool = False):
    """Chunk pooling + scores + selection of the uniform path -> (bits_q, bits_k)
    (+ dict(qc, kc, scores) of the pooled chunks and their (scaled) scores with
    want_pooled).  q_bits: rows the q pooling counts (None: all); k_bits: key
    validity.  k_weights [seq_k] fp32: per-row key pooling weights (Path B) instead
    of k_bits; col_scale [seq_k/chunk_k] fp32: per-key-chunk score scale."""
    _check_cuda(q_re, k_re, q_bits, k_bits, k_weights, col_scale)
    heads, Sq, D = q_re.shape
    Sk = k_re.shape[1]
    mode = selection_mode(sparsity, cdf_threshold)
    n_qt, n_kt = Sq // 64, Sk // 64
    dev = q_re.device
    for t, n in ((k_weights, seq_k), (col_scale, seq_k // chunk_k)):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < n):
            raise ValueError("k_weights / col_scale must be contiguous fp32 of the key rows / chunks")
    bits_q = torch.empty(heads, n_qt, (n_kt + 31) // 32, dtype=torch.int32, device=dev)
    bits_k = torch.empty(heads, n_kt, (n_qt + 31) // 32, dtype=torch.int32, device=dev)
    ws = _ws(_lib.query("prism_block_select_uniform_workspace_bytes", heads, seq_q // chunk_q,
                        seq_k // chunk_k, D), dev)
    _lib.call("prism_block_select_uniform", _p(q_re), _p(k_re), heads, Sq, Sk, D, seq_q, seq_k,
              chunk_q, chunk_k, _p(q_bits), _p(k_bits), _p(k_weights), _p(col_scale), mode,
              float(sparsity if sparsity is not None else 0.0),
              float(cdf_threshold if cdf_threshold is not None else 0.0), _p(ws), _p(bits_q),
              _p(bits_k), _stream(q_re))
    if want_pooled:
        nq, nk = seq_q // chunk_q, seq_k // chunk_k
        f = ws.view(torch.float32)
        qc = f[:heads * nq * D].view(heads, nq, D)
        kc = f[heads * nq * D:heads * (nq + nk) * D].view(heads, nk, D)
        sc = f[heads * (nq + nk) * D:heads * (nq + nk) * D + heads * nq * nk].view(heads, nq, nk)
        return bits_q, bits_k, dict(qc=qc, kc=kc, scores=sc)
    return bits_q, bits_k


# --------------------------------------------------------- bias rectification
def chunk_scores(qc: torch.Tensor, kc: torch.Tensor) -> torch.Tensor:
    """Raw chunk scores [heads, nq, nk] fp32 of pooled q / k chunks."""
    _check_cuda(qc, kc)
    heads, nq, D = qc.shape
    nk = kc.shape[1]
    out = torch.empty(heads, nq, nk, dtype=torch.float32, device=qc.device)
    _lib.call("prism_chunk_scores", _p(qc), _p(kc), heads, nq, nk, D, _p(out), _stream(qc))
    return out


def correction_stats(scores, bits_q, tile_bits, tq: int, tk: int, sm_scale: float, *,
                     want_nonsel: bool = False, want_a_rect: bool = False):
    """(R, M, nonsel, a_rect) of the bias rectification (see prism_correction_stats)."""
    _check_cuda(scores, bits_q, tile_bits)
    heads, nq, nk = scores.shape
    n_qt, n_kt = bits_q.shape[1], tile_bits.shape[0]
    dev = scores.device
    R = torch.empty(heads, nq, dtype=torch.float32, device=dev)
    M = torch.empty(heads, nq, dtype=torch.float32, device=dev)
    nonsel = (torch.empty(heads, nq, (nk + 63) // 64, dtype=torch.int64, device=dev)
              if want_nonsel else None)
    a_rect = torch.empty(heads, nq, nk, dtype=torch.float32, device=dev) if want_a_rect else None
    _lib.call("prism_correction_stats", _p(scores), heads, nq, nk, tq, tk, _p(bits_q), n_qt, n_kt,
              _p(tile_bits), float(sm_scale), _p(R), _p(M), _p(nonsel), _p(a_rect), _stream(scores))
    return R, M, nonsel, a_rect


def taylor_prep(nonsel, M, tau, n_qt: int, tq: int, nk: int, n_ut: int):
    """(masks [heads, n_qt, n_ut] u64, bits_t [heads, n_qt, ceil(n_ut/32)]) of the pooled-key pass."""
    _check_cuda(nonsel, M, tau)
    heads, nq = M.shape
    dev = M.device
    masks = torch.empty(heads, n_qt, n_ut, dtype=torch.int64, device=dev)
    bits_t = torch.empty(heads, n_qt, (n_ut + 31) // 32, dtype=torch.int32, device=dev)
    _lib.call("prism_taylor_prep", _p(nonsel), _p(M), _p(tau), heads, n_qt, tq, nq, nk, n_ut,
              _p(masks), _p(bits_t), _stream(M))
    return masks, bits_t


def key_log_bias(tile_bits, nk: int, tk: int, n_pad: int, sm_scale: float) -> torch.Tensor:
    _check_cuda(tile_bits)
    out = torch.empty(n_pad, dtype=torch.float32, device=tile_bits.device)
    _lib.call("prism_key_log_bias", _p(tile_bits), nk, tk, n_pad, float(sm_scale), _p(out),
              _stream(tile_bits))
    return out


def rows_to_bf16(x: torch.Tensor, n_pad: int) -> torch.Tensor:
    """fp32 [heads, n, D] -> bf16 [heads, n_pad, D], zero rows past n."""
    _check_cuda(x)
    heads, n, D = x.shape
    xc = x.contiguous()
    out = torch.empty(heads, n_pad, D, dtype=torch.bfloat16, device=x.device)
    _lib.call("prism_rows_to_bf16", _p(xc), heads, n, D, n_pad, _p(out), _stream(x))
    return out


def bsa_fwd_keybias(q_re, k_re, v_re, bits_q, key_masks, key_bias, sm_scale: float):
    """Forward with per-(head, q tile, key tile) key masks and per-key score offsets
    -> (o, lse, o_lo)."""
    _check_cuda(q_re, k_re, v_re, bits_q, key_masks, key_bias)
    D0 = q_re.shape[-1]
    Dk = _kernel_head_dim(D0)
    if Dk != D0:
        o, lse, o_lo = bsa_fwd_keybias(_pad_cols(q_re, Dk), _pad_cols(k_re, Dk), _pad_cols(v_re, Dk),
                                       bits_q, key_masks, key_bias, sm_scale)
        return o[..., :D0].contiguous(), lse, o_lo[..., :D0].contiguous()
    heads, Sq, D = q_re.shape
    Sk = k_re.shape[1]
    o = torch.empty_like(q_re)
    o_lo = torch.empty_like(q_re)
    lse = torch.empty(heads, Sq, dtype=torch.float32, device=q_re.device)
    _lib.call("prism_bsa_fwd_keybias", _p(q_re), _p(k_re), _p(v_re), heads, Sq, Sk, D,
              float(sm_scale), _p(bits_q), _p(key_masks), _p(key_bias), _p(o), _p(o_lo), _p(lse),
              _stream(q_re))
    return o, lse, o_lo


def taylor_merge(o_spa, o_spa_lo, lse_spa, o_t, o_t_lo, lse_t, M, tau, seq_q: int, chunk_q: int,
                 out=None):
    _check_cuda(o_spa, lse_spa, o_t, lse_t, M, tau)
    heads, S, D = o_spa.shape
    out = torch.empty_like(o_spa) if out is None else out
    _lib.call("prism_taylor_merge", _p(o_spa), _p(o_spa_lo), _p(lse_spa), _p(o_t), _p(o_t_lo),
              _p(lse_t), _p(M), _p(tau), heads, S, seq_q, chunk_q, D, _p(out), _stream(o_spa))
    return out


def rectified_contract(a_rect: torch.Tensor, v_cmp: torch.Tensor) -> torch.Tensor:
    """a_rect [heads, nq, nk] fp32 x v_cmp [heads, nk, D] fp32 -> [heads, nq, D] fp32
    (fixed summation order over the key chunks)."""
    _check_cuda(a_rect, v_cmp)
    heads, nq, nk = a_rect.shape
    D = v_cmp.shape[-1]
    a = a_rect.contiguous()
    v = v_cmp.contiguous()
    out = torch.empty(heads, nq, D, dtype=torch.float32, device=a_rect.device)
    _lib.call("prism_rectified_contract", _p(a), _p(v), heads, nq, nk, D, _p(out), _stream(a_rect))
    return out


def rectified_apply(o_spa, o_spa_lo, R, o_ncri, seq_q: int, chunk_q: int, out=None):
    _check_cuda(o_spa, R, o_ncri)
    heads, S, D = o_spa.shape
    out = torch.empty_like(o_spa) if out is None else out
    oc = o_ncri.contiguous()
    _lib.call("prism_rectified_apply", _p(o_spa), _p(o_spa_lo), _p(R), _p(oc), heads, S, seq_q,
              chunk_q, D, _p(out), _stream(o_spa))
    return out


# ------------------------------------------------------------- projections
def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False,
         M: Optional[int] = None, N: Optional[int] = None, K: Optional[int] = None,
         bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
         accumulate: bool = False) -> torch.Tensor:
    """prism_gemm_bf16: C[M, N] (+)= sum_k A(m, k) B(n, k) (+ bias).  a, b: 2D bf16
    tensors with unit column stride; K-major A is [M, K] (a_mn: [K, M]), K-major B is
    [N, K] (b_mn: [K, N]).  M / N / K default to the shapes those layouts imply.
    out: a bf16 [M, N] tensor with unit column stride (allocated when None)."""
    _check_cuda(a, b, bias, out)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("gemm expects bf16 operands")
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("gemm operands need unit column stride")
    M = (a.shape[1] if a_mn else a.shape[0]) if M is None else M
    K = (a.shape[0] if a_mn else a.shape[1]) if K is None else K
    N = (b.shape[1] if b_mn else b.shape[0]) if N is None else N
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    bf = None if bias is None else bias.to(torch.float32).contiguous()
    _lib.call("prism_gemm_bf16", _p(a), a.stride(0), int(a_mn), _p(b), b.stride(0), int(b_mn), M, N, K,
              _p(bf), _p(out), out.stride(0), int(accumulate), _stream(a))
    return out


# --------------------------------------------------------- producer fusion
def norm_rope_pack(x: torch.Tensor, heads: int, P: int, hp: int, S_pack: int, gamma=None,
                   eps: float = 1e-6, rope_ff=None, norm: bool = True):
    """x [S, heads*D] bf16 -> (packed [P, S_pack, hp, D] bf16, rstd [S] fp32 or None);
    rope_ff [S, D/2, 4] fp32 (cos_hi, cos_lo, sin_hi, sin_lo)."""
    _check_cuda(x, gamma, rope_ff)
    S, C = x.shape
    D = C // heads
    if x.stride(1) != 1:
        x = x.contiguous()
    out = torch.empty(P, S_pack, hp, D, dtype=torch.bfloat16, device=x.device)
    rstd = torch.empty(S, dtype=torch.float32, device=x.device) if norm else None
    g = None if gamma is None else gamma.to(torch.float32).contiguous()
    _lib.call("prism_norm_rope_pack", _p(x), x.stride(0), S, S_pack, heads, D, P, hp, _p(g),
              float(eps), _p(rope_ff), int(norm), _p(out), _p(rstd), _stream(x))
    return out, rstd


def norm_rope_pack_bwd(g: torch.Tensor, x, heads: int, S: int, gamma=None, rstd=None, rope_ff=None,
                       norm: bool = True):
    """g [P, S_pack, hp, D] -> (dx [S, heads*D] bf16, dgamma [heads*D] fp32 or None)."""
    _check_cuda(g, x, gamma, rstd, rope_ff)
    P, S_pack, hp, D = g.shape
    gc = g.contiguous()
    dx = torch.empty(S, heads * D, dtype=torch.bfloat16, device=g.device)
    dgamma = torch.empty(heads * D, dtype=torch.float32, device=g.device) if norm else None
    ws = _ws(_lib.query("prism_norm_rope_pack_bwd_workspace_bytes", S, heads, D), g.device) if norm else None
    gm = None if gamma is None else gamma.to(torch.float32).contiguous()
    xs = 0 if x is None else x.stride(0)
    _lib.call("prism_norm_rope_pack_bwd", _p(gc), _p(x), xs, S, S_pack, heads, D, P, hp, _p(gm),
              _p(rstd), _p(rope_ff), int(norm), _p(dx), dx.stride(0), _p(ws), _p(dgamma), _stream(g))
    return dx, dgamma


# --------------------------------------------------------- guided selection
def gather_values(x: torch.Tensor, grid, grid_padded, src_idx: torch.Tensor) -> torch.Tensor:
    """Per-token values [T*H*W] on grid -> fp32 [len(src_idx)] in the chunk order, 0 at padding."""
    _check_cuda(x, src_idx)
    xf = x.reshape(-1).to(torch.float32).contiguous()
    T, H, W = grid
    assert xf.numel() == T * H * W, "values must cover the grid"
    out = torch.empty(src_idx.numel(), dtype=torch.float32, device=x.device)
    _lib.call("prism_gather_values", _p(xf), T, H, W, *grid_padded, _p(src_idx), src_idx.numel(),
              _p(out), _stream(x))
    return out


def variance_density(v_re: torch.Tensor, seq_k: int, chunk, k_bits) -> torch.Tensor:
    """compute_channel_variance_density of chunk-ordered V [heads, Sk, D] -> rho [n_chunks] fp32."""
    _check_cuda(v_re, k_bits)
    heads, Sk, D = v_re.shape
    ct, ch, cw = (int(c) for c in chunk)
    rho = torch.empty(seq_k // (ct * ch * cw), dtype=torch.float32, device=v_re.device)
    _lib.call("prism_variance_density", _p(v_re), heads, Sk, D, seq_k, ct, ch, cw, _p(k_bits),
              _p(rho), _stream(v_re))
    return rho


def audio_saliency(norms_re: torch.Tensor, seq_k: int, chunk_k: int, k_bits) -> torch.Tensor:
    """compute_block_audio_saliency of chunk-ordered fp32 norms -> [n_chunks] fp32."""
    _check_cuda(norms_re, k_bits)
    out = torch.empty(seq_k // chunk_k, dtype=torch.float32, device=norms_re.device)
    _lib.call("prism_audio_saliency", _p(norms_re), seq_k, chunk_k, _p(k_bits), _p(out),
              _stream(norms_re))
    return out


def audio_pool_weights(norms_re: torch.Tensor, seq_k: int, chunk_k: int, k_bits,
                       lambda_w: float) -> torch.Tensor:
    """Path B key pooling weights [seq_k] fp32 (0 on invalid rows)."""
    _check_cuda(norms_re, k_bits)
    out = torch.empty(seq_k, dtype=torch.float32, device=norms_re.device)
    _lib.call("prism_audio_pool_weights", _p(norms_re), seq_k, chunk_k, _p(k_bits),
              float(lambda_w), _p(out), _stream(norms_re))
    return out


def pool_chunks(x_re: torch.Tensor, seq: int, chunk: int, bits=None, weights=None) -> torch.Tensor:
    """Chunk means [heads, seq/chunk, D] fp32 of x_re [heads, S, D] bf16 (masked by
    bits, or the Path B weighted form with weights)."""
    _check_cuda(x_re, bits, weights)
    heads, S, D = x_re.shape
    out = torch.empty(heads, seq // chunk, D, dtype=torch.float32, device=x_re.device)
    _lib.call("prism_pool_chunks", _p(x_re), heads, S, D, seq, chunk, _p(bits), _p(weights), _p(out),
              _stream(x_re))
    return out


def guidance_scale(n_chunks: int, device, *, rho=None, variance_gamma: float = 0.0, saliency=None,
                   audio_gate=None, audio_gamma: float = 0.0, modifier=None) -> torch.Tensor:
    """Per-key-chunk score scale 1 + boost [n_chunks] fp32 (see prism_guidance_scale)."""
    _check_cuda(rho, saliency, audio_gate, modifier)
    out = torch.empty(n_chunks, dtype=torch.float32, device=device)
    _lib.call("prism_guidance_scale", n_chunks, _p(rho), float(variance_gamma), _p(saliency),
              _p(audio_gate), float(audio_gamma), _p(modifier), _p(out), _stream(out))
    return out


# -------------------------------------------------------------- a15/a16
class KernelTimer:
    """CUDA events around the attention kernels while a step runs (measurement
    only: ``set_kernel_timer(KernelTimer())`` before the steps, ``totals_ms()``
    after a synchronize).  With a timer set the backward issues its three stages
    (delta, dK/dV, dQ) as three calls, which launch the same kernels in the same
    order as the one-call form."""

    def __init__(self):
        self.spans = {}

    def mark(self, name, device):
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record(torch.cuda.current_stream(device))
        self.spans.setdefault(name, []).append(ev)
        return ev[1]

    def totals_ms(self):
        return {n: sum(a.elapsed_time(b) for a, b in evs) for n, evs in self.spans.items()}

    def counts(self):
        return {n: len(evs) for n, evs in self.spans.items()}


_timer: Optional[KernelTimer] = None


def set_kernel_timer(timer: Optional[KernelTimer]):
    global _timer
    _timer = timer


def _timed(name, device, fn):
    if _timer is None:
        return fn()
    end = _timer.mark(name, device)
    r = fn()
    end.record(torch.cuda.current_stream(device))
    return r


# The attention kernels are built for head dims 64 and 128.  Head dims 16 and 32 (which
# the reference's contract also accepts, bsa_interface.py:604-605) run on the D = 64
# kernels with zero columns appended: a zero column adds exact zeros to every score and
# produces zero output / gradient columns, which are dropped.  The caller's sm_scale
# (1/sqrt of the real head dim) is passed through unchanged.
_KERNEL_D = {16: 64, 32: 64, 64: 64, 128: 128}


def _pad_cols(x: torch.Tensor, Dk: int) -> torch.Tensor:
    if x is None or x.shape[-1] == Dk:
        return x
    out = x.new_zeros(*x.shape[:-1], Dk)
    out[..., :x.shape[-1]] = x
    return out


def _kernel_head_dim(D: int) -> int:
    if D not in _KERNEL_D:
        raise NotImplementedError(f"prism_b200 attention kernels take head_dim 16, 32, 64 or 128, got {D}")
    return _KERNEL_D[D]


def bsa_fwd(q_re, k_re, v_re, bits_q, tile_bits, sm_scale: float, want_lo: bool = False):
    """Returns (o, lse) or (o, lse, o_lo) with o_lo the bf16 rounding residual of o."""
    _check_cuda(q_re, k_re, v_re)
    D0 = q_re.shape[-1]
    Dk = _kernel_head_dim(D0)
    if Dk != D0:
        r = bsa_fwd(_pad_cols(q_re, Dk), _pad_cols(k_re, Dk), _pad_cols(v_re, Dk), bits_q, tile_bits,
                    sm_scale, want_lo)
        return tuple(t[..., :D0].contiguous() if t.dim() == 3 else t for t in r)
    heads, Sq, D = q_re.shape
    Sk = k_re.shape[1]
    o = torch.empty_like(q_re)
    o_lo = torch.empty_like(q_re) if want_lo else None
    lse = torch.empty(heads, Sq, dtype=torch.float32, device=q_re.device)
    _timed("bsa_fwd", q_re.device, lambda: _lib.call(
        "prism_bsa_fwd_qk", _p(q_re), _p(k_re), _p(v_re), heads, Sq, Sk, D, float(sm_scale),
        _p(bits_q), _p(tile_bits), _p(o), _p(o_lo), _p(lse), _stream(q_re)))
    if want_lo:
        return o, lse, o_lo
    return o, lse


def bsa_bwd(q_re, k_re, v_re, o_re, do_re, lse, bits_q, bits_k, tile_bits, sm_scale: float,
            o_lo=None):
    _check_cuda(q_re, do_re)
    D0 = q_re.shape[-1]
    Dk = _kernel_head_dim(D0)
    if Dk != D0:
        g = bsa_bwd(*(_pad_cols(t, Dk) for t in (q_re, k_re, v_re, o_re, do_re)), lse, bits_q, bits_k,
                    tile_bits, sm_scale, o_lo=_pad_cols(o_lo, Dk))
        return tuple(t[..., :D0].contiguous() for t in g)
    heads, Sq, D = q_re.shape
    Sk = k_re.shape[1]
    dq = torch.empty_like(q_re)
    dk = torch.empty_like(k_re)
    dv = torch.empty_like(v_re)
    ws = _ws(_lib.query("prism_bsa_bwd_workspace_bytes", heads, Sq), q_re.device)
    st, sm = _stream(q_re), float(sm_scale)
    if _timer is not None and Sq == Sk:
        dev = q_re.device
        _timed("bsa_bwd_delta", dev, lambda: _lib.call(
            "prism_bsa_bwd_delta", _p(o_re), _p(o_lo), _p(do_re), heads, Sq, D, _p(ws), st))
        _timed("bsa_bwd_dkdv", dev, lambda: _lib.call(
            "prism_bsa_bwd_dkdv", _p(q_re), _p(k_re), _p(v_re), _p(do_re), _p(lse), _p(ws), heads, Sq,
            D, sm, _p(bits_k), _p(tile_bits), _p(dk), _p(dv), st))
        _timed("bsa_bwd_dq", dev, lambda: _lib.call(
            "prism_bsa_bwd_dq", _p(q_re), _p(k_re), _p(v_re), _p(do_re), _p(lse), _p(ws), heads, Sq, D,
            sm, _p(bits_q), _p(tile_bits), _p(dq), st))
        return dq, dk, dv
    _lib.call("prism_bsa_bwd_qk", _p(q_re), _p(k_re), _p(v_re), _p(o_re), _p(o_lo), _p(do_re),
              _p(lse), heads, Sq, Sk, D, sm, _p(bits_q), _p(bits_k), _p(tile_bits),
              _p(ws), _p(dq), _p(dk), _p(dv), st)
    return dq, dk, dv
