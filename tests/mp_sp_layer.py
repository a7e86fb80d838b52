"""Worker for tests/test_gpu_multi.py (launched by torch.distributed.run, one process
per GPU): the fused SelfAttention layer (prism_b200.producer.fused_self_attention,
uniform attention) at P = 1 on every rank, then under Ulysses SP over NCCL with the
packed all-to-alls; rank 0 compares the gathered SP output and input gradients with
the P = 1 result.  Exit status 0 = agreement."""
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    from prism_b200.communications import sp_chunk_sizes
    from prism_b200.parallel_states import initialize_sequence_parallel
    from prism_b200.producer import fused_self_attention, rope_table

    grid, heads, D = (4, 8, 12), 4, 128
    dim, S = heads * D, 4 * 8 * 12
    attn = dict(sparsity=0.5, cdf_threshold=None, chunk_3d_shape_q=(4, 4, 4), chunk_3d_shape_k=(4, 4, 4))
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(1, S, dim, generator=gen).to(torch.bfloat16).to(dev)
    mk = lambda: (torch.randn(dim, dim, generator=gen) / dim ** 0.5).to(torch.bfloat16).to(dev)
    params = {n: mk() for n in ("q_weight", "k_weight", "v_weight", "o_weight")}
    params.update({n: (0.1 * torch.randn(dim, generator=gen)).to(torch.bfloat16).to(dev)
                   for n in ("q_bias", "k_bias", "v_bias", "o_bias")})
    params["norm_q_weight"] = (1 + 0.1 * torch.randn(dim, generator=gen)).to(dev)
    params["norm_k_weight"] = (1 + 0.1 * torch.randn(dim, generator=gen)).to(dev)
    params["eps"] = 1e-6
    gout = torch.randn(1, S, dim, generator=gen).to(torch.bfloat16).to(dev)
    cs = rope_table(grid, D, device=dev)

    # P = 1 (before the sequence-parallel group exists)
    x1 = x.clone().requires_grad_(True)
    ref = fused_self_attention(x1, cs, params, heads, grid, attention="uniform", **attn)
    ref.backward(gout)

    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    initialize_sequence_parallel()
    sizes = sp_chunk_sizes(S, world)
    r0 = sum(sizes[:rank])
    rows = slice(r0, r0 + sizes[rank])
    xl = x[:, rows].clone().requires_grad_(True)
    out = fused_self_attention(xl, cs[rows].contiguous(), params, heads, grid, attention="uniform",
                               full_seq_len=S, **attn)
    out.backward(gout[:, rows])
    outs = [torch.empty(1, sizes[0], dim, dtype=out.dtype, device=dev) for _ in range(world)]
    grads = [torch.empty_like(o) for o in outs]
    dist.all_gather(outs, out.detach().contiguous())
    dist.all_gather(grads, xl.grad.contiguous())
    ok = True
    if rank == 0:
        got, gx = torch.cat(outs, 1)[:, :S].float(), torch.cat(grads, 1)[:, :S].float()
        rel = lambda a, b: float((a - b).norm() / b.norm())
        e_o, e_g = rel(got, ref.float()), rel(gx, x1.grad.float())
        print(f"sp{world}: output rel-L2 {e_o:.2e}, dx rel-L2 {e_g:.2e}", flush=True)
        ok = e_o <= 5e-3 and e_g <= 1e-2
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(flag.item()))


if __name__ == "__main__":
    main()
