"""Ulysses sequence-parallel plumbing on CPU ranks (gloo, world size 2 and 4):
all_to_all_4D in both directions with uneven shards, its autograd backward,
head padding, all_gather with locally derived sizes, the SP average of the
zone statistics, and failure detection (a rank that dies before a collective
makes its peer's collective fail with an error instead of hanging)."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _worker_a2a(rank, world, port, q):
    try:
        _init(rank, world, port)
        from prism_b200.communications import (all_gather, all_to_all_4D, sp_chunk_sizes,
                                               sp_num_local_real_heads, sp_pad_heads,
                                               sp_pad_num_heads)
        from prism_b200 import parallel_states as ps
        ps.initialize_sequence_parallel()
        g = torch.Generator().manual_seed(0)
        S, H, D = 13, 6 if world == 2 else 8, 5
        full = torch.randn(1, S, H, D, generator=g)
        sizes = sp_chunk_sizes(S, world)
        s0 = sum(sizes[:rank])
        shard = full[:, s0:s0 + sizes[rank]].clone().requires_grad_(True)
        group = ps.nccl_info.sp_group
        out = all_to_all_4D(shard, group, scatter_dim=2, gather_dim=1, full_seq_len=S)
        hpr = H // world
        assert out.shape == (1, S, hpr, D), out.shape
        assert torch.equal(out, full[:, :, rank * hpr:(rank + 1) * hpr])
        back = all_to_all_4D(out, group, scatter_dim=1, gather_dim=2, full_seq_len=S)
        assert torch.equal(back, shard.detach())
        # autograd: d/dshard of sum(back * w) == w
        w = torch.randn(back.shape, generator=g)
        (back * w).sum().backward()
        assert torch.allclose(shard.grad, w)
        # head padding for heads % world != 0
        Hr = 5
        padded = sp_pad_num_heads(Hr, world)
        x = sp_pad_heads(full[:, s0:s0 + sizes[rank], :Hr], padded)
        y = all_to_all_4D(x, group, 2, 1, S)
        real = sp_num_local_real_heads(Hr, padded, world, rank)
        hp = padded // world
        ref = torch.cat([full[:, :, :Hr], full.new_zeros(1, S, padded - Hr, D)], 2)[:, :, rank * hp:(rank + 1) * hp]
        assert torch.equal(y, ref) and real == max(0, min(Hr - rank * hp, hp))
        # all_gather with uneven sizes
        z = all_gather(full[:, s0:s0 + sizes[rank], 0, 0].unsqueeze(-1), dim=1, group=group,
                       full_seq_len=S)
        assert torch.equal(z.squeeze(-1), full[:, :, 0, 0])
        # SP average of packed zone statistics
        from prism_b200.dynamic_block_shape import _maybe_sp_average
        packed = torch.full((3, 25 * 4), float(rank + 1))
        avg = _maybe_sp_average(packed.clone())
        assert torch.allclose(avg, torch.full_like(packed, (world + 1) / 2))
        # with heads that leave the last rank idle (it joins with zeros), the average
        # is that of the ranks holding real heads
        from prism_b200.communications import HeadGeometry, live_ranks
        Hs = world - 1
        hg = HeadGeometry(world, Hs)
        mine = torch.full((3, 25 * 4), float(rank + 1)) if hg.real_on(rank) else torch.zeros(3, 25 * 4)
        avg = _maybe_sp_average(mine, live_ranks=live_ranks(Hs, world))
        assert live_ranks(Hs, world) == world - 1
        assert torch.allclose(avg, torch.full_like(avg, world / 2)), avg[0, 0]
        # the heads-side result is a view of the receive buffer, and a heads-side
        # tensor stored in a buffer of P * C rows is sent without a copy
        from prism_b200.communications import ShardGeometry, _heads_as_wire
        C = ShardGeometry(world, S).C
        buf = torch.randn(1, world * C, hpr, D, generator=g)
        view = buf[:, :S]
        w = _heads_as_wire(view, world, C)
        assert w is not None and w.data_ptr() == buf.data_ptr() and w.is_contiguous()
        assert torch.equal(w.reshape(world * C, hpr, D), buf[0])
        assert _heads_as_wire(torch.randn(1, S, hpr, D), world, C) is None or world * C == S
        back2 = all_to_all_4D(view, group, scatter_dim=1, gather_dim=2, full_seq_len=S)
        ref2 = all_to_all_4D(view.contiguous().clone(), group, scatter_dim=1, gather_dim=2, full_seq_len=S)
        assert torch.equal(back2, ref2)
        # batch 2 and the negotiated full length (full_seq_len=None)
        xb = torch.randn(2, sizes[rank], H, D, generator=torch.Generator().manual_seed(rank + 7))
        yb = all_to_all_4D(xb, group, 2, 1)
        assert yb.shape == (2, S, hpr, D)
        zb = all_to_all_4D(yb, group, 1, 2, S)
        assert torch.equal(zb, xb)
        dist.barrier()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _worker_fail(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "exit-before-collective"))
            q.close()
            q.join_thread()  # flush the message before the hard exit
            os._exit(0)  # dies between steps, with no collective in flight
        t = torch.ones(4)
        try:
            dist.all_reduce(t)
            q.put((rank, "collective unexpectedly succeeded"))
        except Exception as e:  # noqa: BLE001 -- the failure is the expected outcome
            q.put((rank, f"detected: {type(e).__name__}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(fn, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_all_to_all_gloo(world):
    res = _run(_worker_a2a, world)
    for r, msg in res.items():
        assert msg == "ok", f"rank {r}: {msg}"


def test_rank_failure_is_detected_not_hung():
    res = _run(_worker_fail, 2)
    assert res[1] == "exit-before-collective"
    assert res[0].startswith("detected"), res[0]
