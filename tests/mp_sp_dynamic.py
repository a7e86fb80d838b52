"""Worker for tests/test_gpu_multi.py (torch.distributed.run, one process per GPU):
the dynamic block-shape attention layer (prism_b200.attention.dynamic_self_attention:
audio-norm all-gather, sequence -> heads exchange, zone statistics averaged over the
SP group, shape choice, selection, sparse attention, heads -> sequence exchange) at
SP = world size over NCCL against the same layer at SP = 1 on the same seeded
inputs (wan_video_dit.py:739-828, dynamic_block_shape.py:132-151).

Per case:
* every rank runs its shard under SP; the shape ids of all ranks holding real heads
  must be identical (one decision per layer);
* rank 0 runs the layer at SP = 1 and counts the zones whose shape id differs from
  SP's.  SP averages per-rank head means of the zone statistics (the reference's
  AVG all-reduce), in a different order than SP = 1's single mean; when every live
  rank holds the same number of real heads the two agree up to rounding, and the
  count must be zero on these seeds.  With uneven real heads per rank the AVG of
  per-rank means is a different statistic (as in the reference) and the count is
  only reported;
* rank 0 runs SP = 1 again with SP's shape ids: output and input gradients must
  equal the gathered SP results bit for bit (same per-head computation).
Cases: 4 heads on an even split; 3 heads on an odd sequence (head padding, a short
last shard; at 4 ranks one idle rank); 1 head (every rank but the first idle: they
join the statistics all-reduce with zeros, and the average divides by the live
ranks).  Exit status 0 = agreement."""
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

CASES = [
    dict(name="h4_even", heads=4, grid=(9, 20, 24), sparsity=0.75, cdf=0.9),
    dict(name="h3_odd", heads=3, grid=(5, 13, 19), sparsity=0.5, cdf=None),
    dict(name="h1_idle", heads=1, grid=(8, 16, 16), sparsity=None, cdf=0.6),
]


def make_case(c, dev):
    T, H, W = c["grid"]
    S, h, D = T * H * W, c["heads"], 128
    gen = torch.Generator().manual_seed(11 + h)
    Tp, Hp, Wp = ((x + 7) // 8 * 8 for x in (T, H, W))

    def zoned():
        mean = torch.randn(h, Tp // 8, Hp // 8, Wp // 8, D, generator=gen) * 0.5
        m = mean.repeat_interleave(8, 1).repeat_interleave(8, 2).repeat_interleave(8, 3)
        x = m + 0.15 * torch.randn(h, Tp, Hp, Wp, D, generator=gen)
        return x[:, :T, :H, :W].reshape(h, S, D).transpose(0, 1).reshape(1, S, h * D)

    q, k, v = zoned(), zoned(), zoned()
    do = torch.randn(1, S, h * D, generator=gen)
    a2v = torch.randn(1, S, 512, generator=gen) * (0.2 + 1.8 * torch.rand(1, S, 1, generator=gen))
    return {n: t.to(torch.bfloat16).to(dev) for n, t in
            dict(q=q, k=k, v=v, do=do, a2v=a2v).items()}, S


def run_layer(inp, c, S, rows):
    from prism_b200.attention import dynamic_self_attention
    q, k, v = (inp[n][:, rows].clone().requires_grad_(True) for n in ("q", "k", "v"))
    out, ids = dynamic_self_attention(q, k, v, c["grid"], c["heads"],
                                      a2v_bridge_residual=inp["a2v"][:, rows].contiguous(),
                                      full_seq_len=S, method="ivpq", sparsity=c["sparsity"],
                                      cdf_threshold=c["cdf"], return_shape_ids=True)
    out.backward(inp["do"][:, rows])
    return out.detach(), q.grad, k.grad, v.grad, ids


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    from prism_b200.communications import HeadGeometry, ShardGeometry
    from prism_b200.parallel_states import (initialize_sequence_parallel, reset_sequence_parallel,
                                            set_sequence_parallel_state)

    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    initialize_sequence_parallel()
    ok = True
    for c in CASES:
        inp, S = make_case(c, dev)
        g = ShardGeometry(world, S)
        hg = HeadGeometry(world, c["heads"])
        rows = slice(g.start(rank), g.start(rank) + g.rows(rank))
        out, dq, dk, dv, ids = run_layer(inp, c, S, rows)
        # one shape decision per layer: every live rank's ids equal rank 0's
        ids0 = ids.clone() if rank == 0 else torch.empty(0, dtype=torch.int64, device=dev)
        n = torch.tensor([ids.numel() if rank == 0 else 0], device=dev)
        dist.broadcast(n, 0)
        if rank != 0:
            ids0 = torch.empty(int(n.item()), dtype=torch.int64, device=dev)
        dist.broadcast(ids0, 0)
        rank_diff = torch.tensor([0 if ids is None else int((ids != ids0).sum().item())], device=dev)
        dist.all_reduce(rank_diff)
        res = []
        for t in (out, dq, dk, dv):
            pad = torch.zeros(1, g.C, t.shape[2], dtype=t.dtype, device=dev)
            pad[:, :t.shape[1]] = t
            parts = torch.empty(world, 1, g.C, t.shape[2], dtype=t.dtype, device=dev)
            dist.all_gather_into_tensor(parts, pad)
            res.append(parts.transpose(0, 1).reshape(1, world * g.C, -1)[:, :S])
        if rank == 0:
            set_sequence_parallel_state(False)
            *_, ids1 = run_layer(inp, c, S, slice(0, S))
            from prism_b200.attention import dynamic_self_attention
            q, k, v = (inp[nm].clone().requires_grad_(True) for nm in ("q", "k", "v"))
            o1 = dynamic_self_attention(q, k, v, c["grid"], c["heads"],
                                        a2v_bridge_residual=inp["a2v"], full_seq_len=S,
                                        method="ivpq", sparsity=c["sparsity"],
                                        cdf_threshold=c["cdf"], shape_ids=ids0)
            o1.backward(inp["do"])
            set_sequence_parallel_state(True)
            even = len({hg.real_on(r) for r in range(world) if hg.real_on(r) > 0}) == 1
            sp1_diff = int((ids1 != ids0).sum().item())
            errs = []
            for name, got, want in zip(("O", "dQ", "dK", "dV"), res,
                                       (o1.detach(), q.grad, k.grad, v.grad)):
                a, b = got.float(), want.float()
                mx = float((a - b).abs().max())
                errs.append(f"{name} max-abs {mx:.2e}")
                ok = ok and torch.equal(got, want)
            print(f"sp{world} {c['name']}: ranks disagreeing on a shape id {int(rank_diff.item())}; "
                  f"zones whose id differs from SP=1's {sp1_diff} of {ids0.numel()} "
                  f"({'must be 0' if even else 'uneven heads per rank: reported'}); "
                  f"vs SP=1 on SP's ids: " + "; ".join(errs), flush=True)
            ok = ok and int(rank_diff.item()) == 0 and (sp1_diff == 0 or not even)
        dist.barrier()
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    reset_sequence_parallel()
    dist.destroy_process_group()
    sys.exit(int(flag.item()))


if __name__ == "__main__":
    main()
