"""The Taylor merge's flat / sharp split under sequence parallelism on CPU ranks (gloo,
world size 2 and 3): global_quantile_across_sp all-gathers every rank's chunk
variances (its head shard) and takes torch.quantile of all of them
(bias_rectification.py:173-187), so every rank gets the same threshold, the one a
single process computes over the concatenation."""
import traceback

import pytest
import torch

from test_sp_gloo import _init, _run


def _worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from prism_b200 import parallel_states as ps
        from prism_b200.bias_rectification import global_quantile_across_sp
        ps.initialize_sequence_parallel()
        g = torch.Generator().manual_seed(3)
        allm = torch.rand(world, 2, 37, generator=g)  # [rank][local heads][q chunks]
        for alpha in (0.5, 0.3, 0.9):
            tau = global_quantile_across_sp(allm[rank], alpha)
            ref = torch.quantile(allm.reshape(-1), alpha)
            assert torch.equal(tau, ref), (alpha, float(tau), float(ref))
            # every rank holds the same threshold
            t = tau.reshape(1).clone()
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            assert torch.equal(t[0], tau)
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_taylor_quantile_across_sp(world):
    res = _run(_worker, world)
    for r, msg in res.items():
        assert msg == "ok", f"rank {r}: {msg}"
