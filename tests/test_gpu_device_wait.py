"""The attention kernels' bounded waits return instead of hanging.

prism_test_fwd_withheld_load runs the forward kernel on one CTA with its producer
issuing no load and the wait limit shortened to 1 ms for that launch: the MMA
warp's first wait can only end at the limit.  The test checks that the call
returns, that the device status reports the wait that gave up (and is cleared by
the read), and that the next normal forward on the same device is correct -- the
CTA released its tensor memory and left nothing in flight.  No fault, trap or
hang is involved: the wait ends on its own limit and the kernel returns."""
import ctypes
import math
import time

import pytest
import torch

from helpers import torch_bsa_reference
from prism_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_withheld_load_times_out_and_device_recovers(cuda):
    L = _lib.load()
    S, D = 256, 128
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, S, D, generator=g).to(torch.bfloat16).to(cuda) for _ in range(3))
    bits_q = torch.full((1, S // 64, 1), 0xF, dtype=torch.int32, device=cuda)  # every pair
    tile_bits = torch.full((S // 64,), -1, dtype=torch.int64, device=cuda)    # every key valid
    o = torch.zeros_like(q)
    lse = torch.zeros(1, S, dtype=torch.float32, device=cuda)
    scale = 1.0 / math.sqrt(D)
    torch.cuda.synchronize()
    assert L.prism_device_status() == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    rc = L.prism_test_fwd_withheld_load(ops._p(q), ops._p(k), ops._p(v), S, D, ctypes.c_float(scale),
                                        ops._p(bits_q), ops._p(tile_bits), ops._p(o), ops._p(lse),
                                        ctypes.c_uint64(1_000_000), stream)
    elapsed = time.perf_counter() - t0
    assert rc == 0, L.prism_last_error()
    code = L.prism_device_status()
    assert code in (102, 103), code          # forward MMA warp or softmax warps gave up
    assert L.prism_device_status() == 0      # the read cleared it
    assert elapsed < 1.0                     # ended at the 1 ms limit, not the default 2 s
    # arguments outside the test entry's limits are refused on the host
    assert L.prism_test_fwd_withheld_load(ops._p(q), ops._p(k), ops._p(v), S, D, ctypes.c_float(scale),
                                          ops._p(bits_q), ops._p(tile_bits), ops._p(o), ops._p(lse),
                                          ctypes.c_uint64(10), stream) != 0
    # the next normal forward on the same device is correct
    o2, lse2 = ops.bsa_fwd(q, k, v, bits_q, tile_bits, scale)
    torch.cuda.synchronize()
    assert L.prism_device_status() == 0
    ref_o, ref_lse, *_ = torch_bsa_reference(q, k, v, torch.zeros_like(q), bits_q, tile_bits, scale)
    assert float((o2.double() - ref_o).abs().max()) <= 2e-2
    assert float((lse2.double() - ref_lse).abs().max()) <= 1e-3
