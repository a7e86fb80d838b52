"""prism_bsa_bwd_noalloc: the sparse-attention backward for callers that may not
allocate device memory while a step runs (engines with a fixed memory plan,
plugins inside a runtime that owns the device pool, code that must not let a
cudaMalloc synchronise the device).  Its only scratch, the per-row delta, is a
fixed array inside the library.

Checked here, through the C ABI: two calls in a row (the second with different
inputs, so stale scratch from the first would show) each match the allocating
entry point prism_bsa_bwd within the suite's tolerance (and in fact bit for
bit: same kernels, same order), and a call beyond the built-in limit is
refused.  This file is collected last so that a failure here leaves every
other test already run; it does not depend on any of them.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from prism_b200 import _lib, ops

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _problem(seed, dev, heads=2, n_tiles=16, D=128, density=0.6):
    g = torch.Generator().manual_seed(seed)
    gd = torch.Generator(device=dev).manual_seed(seed)
    S = n_tiles * 64
    q, k, v, do = (torch.randn(heads, S, D, generator=gd, device=dev).to(torch.bfloat16) for _ in range(4))
    sel = (torch.rand(heads, n_tiles, n_tiles, generator=g) < density).numpy()
    bq = torch.from_numpy(O.dense_to_bits(sel).view(np.int32)).to(dev)
    bk = torch.from_numpy(O.dense_to_bits(sel.transpose(0, 2, 1)).view(np.int32)).to(dev)
    tb = torch.full((n_tiles,), -1, dtype=torch.int64, device=dev)  # every key valid
    return q, k, v, do, bq, bk, tb


def _noalloc(q, k, v, o, o_lo, do, lse, bq, bk, tb, sm):
    heads, S, D = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    p = ops._p
    _lib.call("prism_bsa_bwd_noalloc", p(q), p(k), p(v), p(o), p(o_lo), p(do), p(lse), heads, S, D,
              float(sm), p(bq), p(bk), p(tb), p(dq), p(dk), p(dv), ops._stream(q))
    return dq, dk, dv


def _check(got, ref, what):
    g = got.float().cpu().numpy().astype(np.float64)
    r = ref.float().cpu().numpy().astype(np.float64)
    err = np.abs(g - r).max()
    rel = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
    assert err <= MAX_ABS and rel <= REL_L2, f"{what}: max-abs {err:.3e} rel-L2 {rel:.3e}"
    assert torch.equal(got, ref), f"{what}: not bit-identical to prism_bsa_bwd"


def test_noalloc_backward_matches_allocating_entry_twice(cuda):
    sm = 1.0 / math.sqrt(128)
    for seed in (11, 12):  # two calls in a row, different data each time
        q, k, v, do, bq, bk, tb = _problem(seed, cuda)
        o, lse, o_lo = ops.bsa_fwd(q, k, v, bq, tb, sm, want_lo=True)
        ref = ops.bsa_bwd(q, k, v, o, do, lse, bq, bk, tb, sm, o_lo=o_lo)
        got = _noalloc(q, k, v, o, o_lo, do, lse, bq, bk, tb, sm)
        torch.cuda.synchronize()
        for name, a, b in zip(("dQ", "dK", "dV"), got, ref):
            _check(a, b, f"{name} (seed {seed})")


def test_noalloc_head_dim_64_at_the_full_scratch(cuda):
    """D = 64 with heads * S equal to the limit: the whole array is used (rows at its
    top included) and the result still equals the allocating entry point's."""
    limit = 4 << 20
    heads, n_tiles = 32, 2048
    assert heads * n_tiles * 64 == limit
    sm = 1.0 / math.sqrt(64)
    q, k, v, do, bq, bk, tb = _problem(13, cuda, heads=heads, n_tiles=n_tiles, D=64, density=0.01)
    o, lse, o_lo = ops.bsa_fwd(q, k, v, bq, tb, sm, want_lo=True)
    ref = ops.bsa_bwd(q, k, v, o, do, lse, bq, bk, tb, sm, o_lo=o_lo)
    got = _noalloc(q, k, v, o, o_lo, do, lse, bq, bk, tb, sm)
    torch.cuda.synchronize()
    for name, a, b in zip(("dQ", "dK", "dV"), got, ref):
        _check(a, b, f"{name} (D=64, {heads} x {n_tiles * 64} rows)")


def test_noalloc_rejects_sizes_beyond_the_builtin_scratch(cuda):
    L = _lib.load()
    heads, S = 64, 128 * 1024  # 8M rows > 4M-row limit; refused before any GPU work
    # null tensors: the size check comes first; were it ever skipped, the null-pointer
    # checks would still refuse the call on the host, with no kernel launched
    rc = L.prism_bsa_bwd_noalloc(*([None] * 7), heads, S, 128, ctypes.c_float(0.1),
                                 *([None] * 6), None)
    assert rc != 0
    assert b"exceed the built-in scratch" in L.prism_last_error()
