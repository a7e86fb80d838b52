"""The self-attention layer's projections on the repository's tensor-core GEMM
(``prism_gemm_bf16``) instead of F.linear / cuBLAS.

* ``linear(x, weight, bias)``: ``self.q / self.k / self.v`` (wan_video_dit.py:699-701),
  y = x W^T + b, and its backward: dx = dy W and dW = dy^T x on the same GEMM
  (MN-major operand forms), db = the column sums of dy.
* ``o_proj_packed(recv, weight, bias, heads, S_local)``: ``self.o`` (:841) on the
  inverse exchange's receive buffer ``recv [P, S_pack, hp, D]`` (source rank p
  holds heads [p*hp, p*hp + hp); padded heads are skipped): one GEMM per source
  rank into the same output, the first with the bias, the others accumulating,
  so the heads -> sequence unpack never materialises.  Backward: per source rank
  the slice of d(recv) and the matching columns of dW.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2, weight, bias):
        ctx.save_for_backward(x2, weight)
        ctx.has_bias = bias is not None
        return ops.gemm(x2, weight, bias=bias)

    @staticmethod
    def backward(ctx, gy):
        x2, weight = ctx.saved_tensors
        gy = gy.contiguous()
        dx = ops.gemm(gy, weight, b_mn=True) if ctx.needs_input_grad[0] else None
        dw = ops.gemm(gy, x2, a_mn=True, b_mn=True) if ctx.needs_input_grad[1] else None
        db = gy.sum(0) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [..., K] bf16 (rows contiguous) -> [..., N] bf16 = x W^T + b."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(1) != 1 or x2.stride(0) != x2.shape[1]:
        x2 = x2.contiguous()
    return _Linear.apply(x2, weight, bias).view(*lead, weight.shape[0])


def _source_blocks(P: int, hp: int, heads: int):
    for p in range(P):
        h0, h1 = p * hp, min(p * hp + hp, heads)
        if h1 > h0:
            yield p, h0, h1


class _PackedOProj(torch.autograd.Function):
    @staticmethod
    def forward(ctx, recv, weight, bias, heads, S_local):
        P, S_pack, hp, D = recv.shape
        n_out = weight.shape[0]
        out = torch.empty(S_local, n_out, dtype=torch.bfloat16, device=recv.device)
        rows = recv.view(P, S_pack, hp * D)
        first = True
        for p, h0, h1 in _source_blocks(P, hp, heads):
            ops.gemm(rows[p, :S_local], weight[:, h0 * D:h1 * D], K=(h1 - h0) * D,
                     bias=bias if first else None, out=out, accumulate=not first)
            first = False
        if first:  # no real head anywhere: the bias alone
            out.copy_(bias.expand(S_local, n_out) if bias is not None else torch.zeros_like(out))
        ctx.save_for_backward(recv, weight)
        ctx.meta = (heads, S_local, bias is not None)
        return out

    @staticmethod
    def backward(ctx, gout):
        recv, weight = ctx.saved_tensors
        heads, S_local, has_bias = ctx.meta
        P, S_pack, hp, D = recv.shape
        gout = gout.contiguous()
        rows = recv.view(P, S_pack, hp * D)
        grecv = torch.zeros_like(recv) if ctx.needs_input_grad[0] else None
        dw = torch.zeros_like(weight) if ctx.needs_input_grad[1] else None
        for p, h0, h1 in _source_blocks(P, hp, heads):
            w = weight[:, h0 * D:h1 * D]
            if grecv is not None:
                ops.gemm(gout, w, b_mn=True, out=grecv.view(P, S_pack, hp * D)[p, :S_local, :(h1 - h0) * D])
            if dw is not None:
                ops.gemm(gout, rows[p, :S_local, :(h1 - h0) * D], a_mn=True, b_mn=True, out=dw[:, h0 * D:h1 * D])
        db = gout.sum(0) if has_bias and ctx.needs_input_grad[2] else None
        return grecv, dw, db, None, None


def o_proj_packed(recv: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], heads: int,
                  S_local: int) -> torch.Tensor:
    """self.o of the rows held in recv [P, S_pack, hp, D] (padded heads dropped):
    [S_local, dim_out] bf16."""
    return _PackedOProj.apply(recv.contiguous(), weight, bias, heads, S_local)


__all__ = ["linear", "o_proj_packed"]
