"""Ulysses sequence-parallel collectives around the attention call.

Same names, argument meaning and shard bookkeeping as the reference's
``hymm/utils/communications.py``:

* ``sp_chunk_sizes`` / ``sp_split`` / ``assert_sp_splittable`` (:28-52):
  ``torch.chunk`` shard sizes, the last rank may be shorter;
* ``sp_pad_num_heads`` / ``sp_pad_heads`` / ``sp_num_local_real_heads``
  (:80-110): zero head padding when heads % sp != 0;
* ``all_to_all_4D`` (:134-284): sequence <-> heads reshard with one
  ``all_to_all_single`` per call on the current stream, autograd backward =
  the inverse reshard;
* ``all_gather`` (:346-413) with locally derived shard sizes.

The wire format is the reference's: the send buffer is ``[P, S/P, B, H/P, D]``
(scatter 2 -> gather 1) or ``[P, H/P, S/P, B, D]`` (scatter 1 -> gather 2), so a
rank running this module exchanges byte-identical buffers with a rank running
the reference.  Pack and unpack are single strided copies on the GPU.
"""
from __future__ import annotations

from typing import Any, List, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F


def sp_chunk_sizes(total: int, world_size: int) -> List[int]:
    chunk = (total + world_size - 1) // world_size
    return [min(chunk, max(total - i * chunk, 0)) for i in range(world_size)]


def assert_sp_splittable(total: int, world_size: int, name: str = "sequence"):
    if world_size <= 1:
        return
    sizes = sp_chunk_sizes(total, world_size)
    assert sizes[-1] > 0, (
        f"{name} length {total} is too short for sp_size={world_size}: the trailing SP rank(s) "
        f"would receive zero tokens.")


def sp_split(x: torch.Tensor, world_size: int, rank: int, dim: int) -> torch.Tensor:
    if world_size <= 1:
        return x
    sizes = sp_chunk_sizes(x.shape[dim], world_size)
    return torch.split(x, sizes, dim=dim)[rank]


def sp_pad_num_heads(num_heads: int, sp_size: int) -> int:
    r = num_heads % sp_size
    return num_heads if r == 0 else num_heads + (sp_size - r)


def sp_pad_heads(x: torch.Tensor, padded_heads: int, dim: int = 2) -> torch.Tensor:
    cur = x.shape[dim]
    if cur >= padded_heads:
        return x
    shape = list(x.shape)
    shape[dim] = padded_heads - cur
    return torch.cat([x, x.new_zeros(shape)], dim=dim)


def sp_num_local_real_heads(num_real_heads: int, padded_heads: int, sp_size: int, sp_rank: int) -> int:
    hpr = padded_heads // sp_size
    return max(0, min(num_real_heads - sp_rank * hpr, hpr))


def _all_to_all_4D(input: torch.Tensor, scatter_idx: int = 2, gather_idx: int = 1, group=None,
                   full_seq_len: Optional[int] = None) -> torch.Tensor:
    assert input.dim() == 4, f"input must be 4D tensor, got {input.dim()}"
    P = dist.get_world_size(group)
    rank = dist.get_group_rank(group, dist.get_rank())
    if scatter_idx == 2 and gather_idx == 1:
        # (bs, S/P, hc, hs) -> (bs, S, hc/P, hs)
        if full_seq_len is not None:
            sizes = sp_chunk_sizes(int(full_seq_len), P)
        else:
            sizes = [None] * P
            dist.all_gather_object(sizes, input.shape[1], group)
        gap = sizes[0] - sizes[-1]
        if gap > 0 and rank == P - 1:
            input = F.pad(input, (0, 0, 0, 0, 0, gap))
        bs, shard, hc, hs = input.shape
        assert hc % P == 0, f"Invalid Head size: {hc}, which should be divisible by spsize {P}"
        shc = hc // P
        send = input.reshape(bs, shard, P, shc, hs).permute(2, 1, 0, 3, 4).contiguous()
        if P > 1:
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=group)
        else:
            recv = send
        out = recv.reshape(P * shard, bs, shc, hs).transpose(0, 1).contiguous()
        if gap > 0:
            out = out[:, : P * shard - gap]
        return out
    if scatter_idx == 1 and gather_idx == 2:
        # (bs, S, hc/P, hs) -> (bs, S/P, hc, hs)
        bs, S, shc, hs = input.shape
        hc = shc * P
        gap = 0
        if S % P != 0:
            gap = (S // P + 1) * P - S
            input = F.pad(input, (0, 0, 0, 0, 0, gap))
            S = S + gap
        shard = S // P
        send = input.reshape(bs, P, shard, shc, hs).permute(1, 3, 2, 0, 4).contiguous()
        if P > 1:
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=group)
        else:
            recv = send
        out = recv.reshape(hc, shard, bs, hs).permute(2, 1, 0, 3).contiguous()
        if gap > 0 and rank == P - 1:
            out = out[:, :-gap]
        return out
    raise RuntimeError("scatter_idx must be 1 or 2 and gather_idx must be 1 or 2")


class SeqAllToAll4D(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, group, input, scatter_idx, gather_idx, full_seq_len=None):
        ctx.group = group
        ctx.scatter_idx = scatter_idx
        ctx.gather_idx = gather_idx
        ctx.full_seq_len = full_seq_len
        return _all_to_all_4D(input, scatter_idx, gather_idx, group=group, full_seq_len=full_seq_len)

    @staticmethod
    def backward(ctx: Any, *grad_output):
        return (None,
                SeqAllToAll4D.apply(ctx.group, *grad_output, ctx.gather_idx, ctx.scatter_idx,
                                    ctx.full_seq_len),
                None, None, None)


def all_to_all_4D(input_: torch.Tensor, group, scatter_dim: int = 2, gather_dim: int = 1,
                  full_seq_len: Optional[int] = None):
    return SeqAllToAll4D.apply(group, input_, scatter_dim, gather_dim, full_seq_len)


class _AllGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input_, dim, group, full_seq_len=None):
        world = dist.get_world_size(group)
        rank = dist.get_group_rank(group, dist.get_rank())
        if full_seq_len is not None:
            sizes = sp_chunk_sizes(int(full_seq_len), world)
        else:
            shapes = [None] * world
            dist.all_gather_object(shapes, input_.shape[dim], group)
            sizes = [int(s) for s in shapes]
        ctx.dim, ctx.group, ctx.sizes, ctx.rank = dim, group, sizes, rank
        input_ = input_.contiguous()
        if all(s == sizes[0] for s in sizes):
            if dim == 0:
                shape = list(input_.shape)
                shape[0] = sizes[0] * world
                flat = torch.empty(shape, dtype=input_.dtype, device=input_.device)
                dist.all_gather_into_tensor(flat, input_, group=group)
                return flat
            lst = [torch.empty_like(input_) for _ in range(world)]
            dist.all_gather(lst, input_, group=group)
            return torch.cat(lst, dim=dim)
        # ragged shards: pad to the largest shard, one uniform all-gather, slice
        # (the reference issues a ragged dist.all_gather, i.e. one broadcast per rank)
        mx = max(sizes)
        pad = mx - input_.shape[dim]
        if pad > 0:
            shape = list(input_.shape)
            shape[dim] = pad
            input_ = torch.cat([input_, input_.new_zeros(shape)], dim=dim)
        lst = [torch.empty_like(input_) for _ in range(world)]
        dist.all_gather(lst, input_, group=group)
        return torch.cat([t.narrow(dim, 0, s) for t, s in zip(lst, sizes)], dim=dim)

    @staticmethod
    def backward(ctx, grad_output):
        g = torch.split(grad_output, ctx.sizes, dim=ctx.dim)[ctx.rank]
        return g.contiguous(), None, None, None


def all_gather(input_: torch.Tensor, dim: int = 1, group=None, full_seq_len: Optional[int] = None):
    return _AllGather.apply(input_, dim, group, full_seq_len)


__all__ = [
    "sp_chunk_sizes", "assert_sp_splittable", "sp_split", "sp_pad_num_heads", "sp_pad_heads",
    "sp_num_local_real_heads", "all_to_all_4D", "SeqAllToAll4D", "all_gather",
]
