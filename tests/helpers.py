"""Shared test helpers: fixture loading and bf16 bit views."""
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 numpy bit pattern."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def load_fixture(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def torch_bsa_reference(q, k, v, do, bits_q, tile_bits, sm_scale, block_rows=1024):
    """Block-sparse attention forward + backward in float64 on the tensors' device:
    dense masked softmax attention restricted to the selected (query tile, key tile)
    pairs and valid keys -- the definition the reference's Triton kernels compute
    (flash_attn_bsa_varlen_mask.py:193-319 forward, 564-704 dK/dV, 881-1014 dQ,
    common.py:94-111 delta).  A test-only checker for grids too large for the numpy
    oracle (test_gpu_config_parity pins it to the oracle on a small case).

    q, k, v, do: [heads, S, D] (tile order); bits_q [heads, S/64, W] int32 bitmaps;
    tile_bits [S/64] int64 key-validity words.  Returns float64 (o, lse, dq, dk, dv);
    rows with no selected valid key get o = 0, lse = -inf and zero gradients."""
    import torch
    heads, S, D = q.shape
    nt = S // 64
    dev = q.device
    shifts = torch.arange(32, device=dev, dtype=torch.int64)
    words = bits_q.to(torch.int64) & 0xFFFFFFFF
    tile_mask = ((words[..., None] >> shifts) & 1).bool().reshape(heads, nt, -1)[:, :, :nt]
    kbits = tile_bits.to(torch.int64)
    sh64 = torch.arange(64, device=dev, dtype=torch.int64)
    kvalid = ((kbits[:, None] >> sh64) & 1).bool().reshape(-1)
    f = lambda t: t.to(torch.float64)
    o = torch.zeros(heads, S, D, dtype=torch.float64, device=dev)
    lse = torch.full((heads, S), float("-inf"), dtype=torch.float64, device=dev)
    dq = torch.zeros_like(o)
    dk = torch.zeros_like(o)
    dv = torch.zeros_like(o)
    for h in range(heads):
        qh, kh, vh, doh = f(q[h]), f(k[h]), f(v[h]), f(do[h])
        for r0 in range(0, S, block_rows):
            r1 = min(S, r0 + block_rows)
            m = tile_mask[h, r0 // 64:(r1 + 63) // 64].repeat_interleave(64, 0)[: r1 - r0]
            m = m.repeat_interleave(64, 1) & kvalid[None, :]
            s = (qh[r0:r1] @ kh.T) * sm_scale
            s.masked_fill_(~m, float("-inf"))
            mx = s.max(1, keepdim=True).values
            live = torch.isfinite(mx)
            p = torch.exp(s - torch.where(live, mx, torch.zeros_like(mx)))
            del s
            l = p.sum(1, keepdim=True)
            p = torch.where(live, p / torch.where(live, l, torch.ones_like(l)), torch.zeros_like(p))
            ob = p @ vh
            o[h, r0:r1] = ob
            lse[h, r0:r1] = torch.where(live, mx + torch.log(l), mx)[:, 0]
            delta = (ob * doh[r0:r1]).sum(1, keepdim=True)
            dp = doh[r0:r1] @ vh.T
            ds = p * (dp - delta)
            del dp
            dq[h, r0:r1] = (ds @ kh) * sm_scale
            dk[h] += (ds.T @ qh[r0:r1]) * sm_scale
            dv[h] += p.T @ doh[r0:r1]
            del p, ds
    return o, lse, dq, dk, dv
