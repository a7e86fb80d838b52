"""Ulysses sequence <-> head exchange around the attention call.

The reference reshards with ``all_to_all_4D`` / ``all_gather``
(hymm/utils/communications.py:134-284, 346-413; callers
wan_video_dit.py:739-787, 824-828).  The public names the DiT imports are kept
(``all_to_all_4D``, ``all_gather``, ``sp_split``, ``sp_chunk_sizes``,
``assert_sp_splittable``, ``sp_pad_num_heads``, ``sp_pad_heads``,
``sp_num_local_real_heads``) with the same argument meaning; the exchange itself
is built around one buffer layout chosen so that the attention side never copies.

Geometry.  A sequence of S tokens is cut into P shards of ``C = ceil(S / P)``
rows; shard r starts at r * C and the last shard may be shorter (a rank whose
shard would be empty is an error).  H heads are padded to ``P * hp`` with
``hp = ceil(H / P)`` heads per rank; rank r owns heads [r * hp, r * hp + hp).

Wire layout.  Both directions exchange ``[P, B, C, hp, D]`` buffers with one
``all_to_all_single``: block p of a send buffer goes to rank p.
* heads side: block p of rank r's buffer holds tokens [p * C, p * C + C) of
  r's hp heads.  With B = 1 the whole buffer is ``[P * C, hp, D]`` - the full
  sequence of r's heads, token-major - so the attention reads a receive buffer
  in place (``[1, S, hp, D]`` view, no unpack) and its output, written into a
  buffer of P * C rows (``seq_capacity``), is sent as it is (no pack).
* sequence side: block p holds this rank's C rows of heads [p * hp, p * hp + hp).
  Going there from the token-major ``[B, S_local, H, D]`` activations (and back)
  is one strided copy, the only copy per exchange; the fused layer
  (prism_b200.producer) removes it as well by writing and reading this layout
  directly.  Rows past a short last shard travel as filler and are dropped.

Everything runs on the current CUDA stream (NCCL) or on CPU tensors (gloo).
Collectives carry no timeout handling of their own: a rank that misses one makes
its peers fail through the process group's timeout, not hang silently.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist


# ----------------------------------------------------------------- geometry
@dataclass(frozen=True)
class ShardGeometry:
    """P shards of a sequence of S tokens, C = ceil(S / P) rows each (last shorter)."""

    P: int
    S: int

    @property
    def C(self) -> int:
        return -(-self.S // self.P)

    def start(self, r: int) -> int:
        return min(r * self.C, self.S)

    def rows(self, r: int) -> int:
        return max(0, min(self.C, self.S - r * self.C))


@dataclass(frozen=True)
class HeadGeometry:
    """H real heads over P ranks, hp = ceil(H / P) per rank (tail heads are padding)."""

    P: int
    H: int

    @property
    def hp(self) -> int:
        return -(-self.H // self.P)

    def real_on(self, r: int) -> int:
        return max(0, min(self.hp, self.H - r * self.hp))


def sp_chunk_sizes(total: int, world_size: int) -> List[int]:
    """Shard lengths of a sequence of ``total`` tokens over ``world_size`` ranks."""
    g = ShardGeometry(int(world_size), int(total))
    return [g.rows(r) for r in range(g.P)]


def assert_sp_splittable(total: int, world_size: int, name: str = "sequence"):
    """Every rank must receive at least one token (an empty shard cannot join the exchange)."""
    if world_size > 1:
        g = ShardGeometry(int(world_size), int(total))
        assert g.rows(g.P - 1) > 0, (
            f"{name}: {total} tokens over {world_size} SP ranks leaves rank {world_size - 1} "
            f"without tokens (shards of {g.C})")


def sp_split(x: torch.Tensor, world_size: int, rank: int, dim: int) -> torch.Tensor:
    """This rank's shard of ``x`` along ``dim`` (a view)."""
    if world_size <= 1:
        return x
    g = ShardGeometry(int(world_size), x.shape[dim])
    return x.narrow(dim, g.start(rank), g.rows(rank))


def sp_pad_num_heads(num_heads: int, sp_size: int) -> int:
    """Head count after padding to a multiple of the SP size."""
    g = HeadGeometry(int(sp_size), int(num_heads))
    return g.hp * g.P


def sp_pad_heads(x: torch.Tensor, padded_heads: int, dim: int = 2) -> torch.Tensor:
    """Zero heads appended along ``dim`` up to ``padded_heads``."""
    n = x.shape[dim]
    if n >= padded_heads:
        return x
    shape = list(x.shape)
    shape[dim] = padded_heads
    out = x.new_zeros(shape)
    out.narrow(dim, 0, n).copy_(x)
    return out


def sp_num_local_real_heads(num_real_heads: int, padded_heads: int, sp_size: int,
                            sp_rank: int) -> int:
    """Real (non-padding) heads among the ``padded_heads / sp_size`` heads of ``sp_rank``."""
    hp = padded_heads // sp_size
    return max(0, min(hp, num_real_heads - sp_rank * hp))


def live_ranks(num_real_heads: int, sp_size: int) -> int:
    """Ranks that hold at least one real head."""
    g = HeadGeometry(int(sp_size), int(num_real_heads))
    return sum(1 for r in range(g.P) if g.real_on(r) > 0)


# ------------------------------------------------------------ group helpers
def _group_info(group):
    return dist.get_world_size(group), dist.get_group_rank(group, dist.get_rank())


def _negotiate_length(local: int, P: int, group, device) -> int:
    """Full sequence length from every rank's shard length; the shards must follow
    ShardGeometry (the wire layout assumes it)."""
    mine = torch.tensor([int(local)], dtype=torch.int64, device=device)
    every = torch.empty(P, dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(every, mine, group=group)
    lens = [int(x) for x in every.tolist()]
    S = sum(lens)
    if lens != sp_chunk_sizes(S, P):
        raise ValueError(f"shard lengths {lens} are not the ceil(S/P) split of {S} tokens")
    return S


def _timed_span(name: str, x: torch.Tensor, fn):
    """fn() inside a CUDA-event span of the step timer (prism_b200.ops.KernelTimer)
    when one is set (CUDA tensors only; measurement, not part of the exchange)."""
    if x.is_cuda:
        from . import ops
        return ops._timed(name, x.device, fn)
    return fn()


def _exchange(send: torch.Tensor, group, P: int) -> torch.Tensor:
    """One all_to_all_single over dim 0 of a contiguous [P, ...] buffer."""
    if P == 1:
        return send
    recv = torch.empty_like(send)
    _timed_span("sp_all_to_all", send, lambda: dist.all_to_all_single(recv, send, group=group))
    return recv


# ------------------------------------------------------ layout conversions
def _row_copy_ok(*ts) -> bool:
    """The row-copy kernel (prism_copy_rows) applies: CUDA tensors, 16-byte aligned
    storage offsets and rows (a rank's hp heads of one token) of whole 16-byte chunks."""
    return all(t.is_cuda and t.data_ptr() % 16 == 0 and t.stride(-1) == 1 for t in ts)


def _seq_to_wire(x: torch.Tensor, P: int, C: int, hp: int) -> torch.Tensor:
    """[B, S_local, P*hp, D] (token-major) -> contiguous wire [P, B, C, hp, D]."""
    B, n, Hp, D = x.shape
    wire = x.new_empty(P, B, C, hp, D)
    es = x.element_size()
    if (B == 1 and x.stride(2) == D and (hp * D * es) % 16 == 0 and (x.stride(1) * es) % 16 == 0
            and _row_copy_ok(x, wire)):
        # block p = heads [p hp, p hp + hp) of every token: one contiguous hp*D row per token
        from . import ops
        ops.copy_rows(x, (hp * D, x.stride(1)), wire, (C * hp * D, hp * D), P, n, hp * D)
    else:
        wire[:, :, :n].copy_(x.unflatten(2, (P, hp)).permute(2, 0, 1, 3, 4))
    if n < C:
        wire[:, :, n:].zero_()
    return wire


def _wire_to_seq(wire: torch.Tensor, n: int) -> torch.Tensor:
    """Wire [P, B, C, hp, D] -> [B, n, P*hp, D] (this rank's first n rows)."""
    P, B, C, hp, D = wire.shape
    out = wire.new_empty(B, n, P, hp, D)
    es = wire.element_size()
    if B == 1 and wire.is_contiguous() and (hp * D * es) % 16 == 0 and _row_copy_ok(wire, out):
        from . import ops
        ops.copy_rows(wire, (C * hp * D, hp * D), out, (hp * D, P * hp * D), P, n, hp * D)
    else:
        out.copy_(wire[:, :, :n].permute(1, 2, 0, 3, 4))
    return out.view(B, n, P * hp, D)


def _heads_as_wire(x: torch.Tensor, P: int, C: int) -> Optional[torch.Tensor]:
    """A [1, S, hp, D] token-major tensor whose storage extends to P*C rows, viewed
    as the wire [P, 1, C, hp, D] without a copy (None if it does not qualify).
    The rows past S are filler: the receiver of that block drops them."""
    B, S, hp, D = x.shape
    if B != 1 or not x[0].is_contiguous():
        return None
    need = (x.storage_offset() + P * C * hp * D) * x.element_size()
    if x.untyped_storage().nbytes() < need:
        return None
    return x.as_strided((P, 1, C, hp, D), (C * hp * D, P * C * hp * D, hp * D, D, 1),
                        x.storage_offset())


def _heads_to_wire(x: torch.Tensor, P: int, C: int) -> torch.Tensor:
    """[B, S, hp, D] (full sequence of this rank's heads) -> wire [P, B, C, hp, D]
    (a view of x when _heads_as_wire qualifies it, else one copy)."""
    w = _heads_as_wire(x, P, C)
    if w is not None:
        return w
    B, S, hp, D = x.shape
    full = x.new_empty(B, P * C, hp, D)
    full[:, :S].copy_(x)
    if S < P * C:
        full[:, S:].zero_()
    return full.view(B, P, C, hp, D).permute(1, 0, 2, 3, 4)


def _wire_to_heads(wire: torch.Tensor, S: int) -> torch.Tensor:
    """Wire [P, B, C, hp, D] -> [B, S, hp, D]: a view for B = 1."""
    P, B, C, hp, D = wire.shape
    if B == 1:
        return wire.view(1, P * C, hp, D)[:, :S]
    return wire.permute(1, 0, 2, 3, 4).reshape(B, P * C, hp, D)[:, :S]


# ------------------------------------------------------- autograd functions
def _seq_to_heads(x, group, S):
    P, r = _group_info(group)
    g = ShardGeometry(P, S)
    B, n, Hp, D = x.shape
    if Hp % P:
        raise ValueError(f"{Hp} heads do not split over {P} SP ranks; pad them first (sp_pad_heads)")
    if n != g.rows(r):
        raise ValueError(f"rank {r} holds {n} tokens, the split of {S} over {P} gives {g.rows(r)}")
    wire = _timed_span("sp_layout_copy", x, lambda: _seq_to_wire(x, P, g.C, Hp // P))
    recv = _exchange(wire, group, P)
    return _wire_to_heads(recv, S)


def _heads_to_seq(x, group, S):
    P, r = _group_info(group)
    g = ShardGeometry(P, S)
    if x.shape[1] != S:
        raise ValueError(f"expected the full sequence of {S} tokens, got {x.shape[1]}")
    wire = _timed_span("sp_layout_copy", x, lambda: _heads_to_wire(x, P, g.C).contiguous())
    recv = _exchange(wire, group, P)
    return _timed_span("sp_layout_copy", recv, lambda: _wire_to_seq(recv, g.rows(r)))


class SeqToHeads(torch.autograd.Function):
    """[B, S_local, H, D] -> [B, S, H/P, D]; the backward is the inverse exchange."""

    @staticmethod
    def forward(ctx, x, group, S):
        ctx.group, ctx.S = group, S
        return _seq_to_heads(x, group, S)

    @staticmethod
    def backward(ctx, g):
        return _heads_to_seq(g, ctx.group, ctx.S), None, None


class HeadsToSeq(torch.autograd.Function):
    """[B, S, H/P, D] -> [B, S_local, H, D]; the backward is the inverse exchange."""

    @staticmethod
    def forward(ctx, x, group, S):
        ctx.group, ctx.S = group, S
        return _heads_to_seq(x, group, S)

    @staticmethod
    def backward(ctx, g):
        return _seq_to_heads(g, ctx.group, ctx.S), None, None


class WireToHeads(torch.autograd.Function):
    """A sequence-side wire buffer [P, B, C, hp, D] that a producer wrote directly
    (prism_norm_rope_pack) -> exchange -> [B, S, hp, D] (a view of the receive
    buffer for B = 1).  Backward: the heads-side gradient is sent back (without a
    copy when it lives in a buffer of P * C rows) and arrives as the wire's gradient."""

    @staticmethod
    def forward(ctx, wire, group, S):
        P, _ = _group_info(group)
        ctx.group, ctx.P, ctx.C = group, P, wire.shape[2]
        return _wire_to_heads(_exchange(wire.contiguous(), group, P), S)

    @staticmethod
    def backward(ctx, g):
        return _exchange(_heads_to_wire(g, ctx.P, ctx.C).contiguous(), ctx.group, ctx.P), None, None


class HeadsToWire(torch.autograd.Function):
    """[B, S, hp, D] -> exchange -> the sequence-side receive buffer [P, B, C, hp, D]
    for a consumer that reads that layout directly (the K-split output projection).
    The input is sent without a copy when it lives in a buffer of P * C rows."""

    @staticmethod
    def forward(ctx, x, group, S):
        P, _ = _group_info(group)
        C = ShardGeometry(P, S).C
        ctx.group, ctx.P, ctx.S = group, P, S
        return _exchange(_heads_to_wire(x, P, C).contiguous(), group, P)

    @staticmethod
    def backward(ctx, g):
        return _wire_to_heads(_exchange(g.contiguous(), ctx.group, ctx.P), ctx.S), None, None


def all_to_all_4D(input_: torch.Tensor, group, scatter_dim: int = 2, gather_dim: int = 1,
                  full_seq_len: Optional[int] = None):
    """scatter_dim=2, gather_dim=1: [B, S/P, H, D] -> [B, S, H/P, D] (sequence to heads);
    scatter_dim=1, gather_dim=2: the inverse.  ``full_seq_len`` is S (negotiated over
    the group when None).  Differentiable; the result of the forward direction is a
    view of the receive buffer."""
    if input_.dim() != 4:
        raise ValueError(f"all_to_all_4D expects a 4D tensor, got {input_.dim()}D")
    P, _ = _group_info(group)
    if (scatter_dim, gather_dim) == (2, 1):
        S = full_seq_len if full_seq_len is not None else _negotiate_length(
            input_.shape[1], P, group, input_.device)
        return SeqToHeads.apply(input_, group, int(S))
    if (scatter_dim, gather_dim) == (1, 2):
        S = input_.shape[1] if full_seq_len is None else int(full_seq_len)
        return HeadsToSeq.apply(input_, group, int(S))
    raise ValueError("all_to_all_4D supports (scatter_dim, gather_dim) = (2, 1) or (1, 2)")


class _GatherSequence(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, group, S):
        P, r = _group_info(group)
        g = ShardGeometry(P, S)
        if x.shape[dim] != g.rows(r):
            raise ValueError(f"rank {r} holds {x.shape[dim]} rows, the split of {S} gives {g.rows(r)}")
        ctx.dim, ctx.start, ctx.rows = dim, g.start(r), g.rows(r)
        front = x.movedim(dim, 0)
        slab = front.new_zeros((g.C,) + tuple(front.shape[1:]))
        slab[: g.rows(r)].copy_(front)
        full = slab.new_empty((P * g.C,) + tuple(slab.shape[1:]))
        if P > 1:
            dist.all_gather_into_tensor(full, slab, group=group)
        else:
            full.copy_(slab)
        return full[:S].movedim(0, dim)

    @staticmethod
    def backward(ctx, grad):
        return grad.narrow(ctx.dim, ctx.start, ctx.rows), None, None, None


def all_gather(input_: torch.Tensor, dim: int = 1, group=None, full_seq_len: Optional[int] = None):
    """Concatenate every rank's shard along ``dim`` (shards follow ShardGeometry; S is
    negotiated when ``full_seq_len`` is None).  The backward keeps this rank's rows."""
    P, _ = _group_info(group)
    S = full_seq_len if full_seq_len is not None else _negotiate_length(
        input_.shape[dim], P, group, input_.device)
    return _GatherSequence.apply(input_, dim, group, int(S))


__all__ = [
    "ShardGeometry", "HeadGeometry", "sp_chunk_sizes", "assert_sp_splittable", "sp_split",
    "sp_pad_num_heads", "sp_pad_heads", "sp_num_local_real_heads", "live_ranks", "all_to_all_4D",
    "SeqToHeads", "HeadsToSeq", "WireToHeads", "HeadsToWire", "all_gather",
]
