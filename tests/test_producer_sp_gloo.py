"""The fused layer's Ulysses plumbing on CPU ranks (gloo, world size 2 and 4): the
wire exchanges WireToHeads / HeadsToWire (send layout [P, S_pack, hp, D] as
prism_norm_rope_pack writes it, head padding, an uneven last shard), their autograd
adjoint, and the K-split output projection on the inverse exchange's receive buffer
against the unpacked projection (wan_video_dit.py:775-787, 824-841).  The attention
in between is the identity, so two exchanges bring every rank its own tokens back."""
import traceback

import pytest
import torch

from test_sp_gloo import _init, _run


def _k_split_projection(recv, W, b, heads, S_local):
    """The K-split form prism_b200.linear.o_proj_packed computes on the GPU: the sum
    over source ranks p of recv[p] W[:, heads of p]^T (padded heads skipped), + b."""
    P, S_pack, hp, D = recv.shape
    out = b.expand(S_local, W.shape[0]).clone()
    for p in range(P):
        h0, h1 = p * hp, min(p * hp + hp, heads)
        if h1 > h0:
            out = out + recv[p, :S_local, : h1 - h0].reshape(S_local, -1) @ W[:, h0 * D:h1 * D].t()
    return out


def _worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from prism_b200 import parallel_states as ps
        from prism_b200.communications import sp_chunk_sizes, sp_pad_num_heads
        from prism_b200.communications import HeadsToWire, WireToHeads
        ps.initialize_sequence_parallel()
        group = ps.nccl_info.sp_group
        g = torch.Generator().manual_seed(0)
        S, H, D = 13, 6, 4
        full = torch.randn(S, H, D, generator=g, dtype=torch.float64)
        W = torch.randn(7, H * D, generator=g, dtype=torch.float64)
        b = torch.randn(7, generator=g, dtype=torch.float64)
        sizes = sp_chunk_sizes(S, world)
        S_pack = sizes[0]
        s0 = sum(sizes[:rank])
        mine = full[s0:s0 + sizes[rank]]
        padded = sp_pad_num_heads(H, world)
        hp = padded // world
        # the producer's send layout: send[p, s, hh] = token s, head p * hp + hh
        send = torch.zeros(world, S_pack, hp, D, dtype=torch.float64)
        for p in range(world):
            for hh in range(hp):
                h = p * hp + hh
                if h < H:
                    send[p, :sizes[rank], hh] = mine[:, h]
        send.requires_grad_(True)
        seq4 = WireToHeads.apply(send.unsqueeze(1), group, S)   # [1, S, hp, D]
        seq = seq4[0]                                           # the full sequence, my heads
        for hh in range(hp):
            h = rank * hp + hh
            want = full[:, h] if h < H else torch.zeros(S, D, dtype=torch.float64)
            assert torch.equal(seq[:, hh], want), (rank, hh)
        # inverse exchange of the (identity) attention output, then the K-split projection
        recv2 = HeadsToWire.apply(seq4, group, S).squeeze(1)    # [P, S_pack, hp, D]
        out = _k_split_projection(recv2, W, b, H, sizes[rank])
        ref = mine.reshape(sizes[rank], H * D) @ W.t() + b
        assert torch.allclose(out, ref, rtol=1e-12, atol=1e-12)
        # adjoint: the gradient of sum(out * w) reaches the send buffer's real entries as
        # the unpacked projection's gradient, and zero on padding
        w = torch.randn(out.shape, generator=g, dtype=torch.float64)
        (out * w).sum().backward()
        gref = (w @ W).reshape(sizes[rank], H, D)
        for p in range(world):
            for hh in range(hp):
                h = p * hp + hh
                gs = send.grad[p, :sizes[rank], hh]
                assert torch.allclose(gs, gref[:, h] if h < H else torch.zeros_like(gs)), (p, hh)
            assert not send.grad[p, sizes[rank]:].any()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4])
def test_packed_all_to_all_and_k_split_projection(world):
    res = _run(_worker, world)
    for r, msg in res.items():
        assert msg == "ok", f"rank {r}: {msg}"
