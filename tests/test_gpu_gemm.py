"""The tensor-core GEMM of the layer's projections (prism_gemm_bf16) against a
float32 product of the same bf16 operands, in its three operand layouts (forward
y = x W^T, dgrad dx = dy W, wgrad dW = dy^T x), with partial tiles in every
dimension, a bias, the accumulate form and a strided output; run-to-run
bit-identical.  Tolerance: bf16 output rounding (relative L2 4e-3, max-abs 1e-2 of
the output's largest magnitude)."""
import pytest
import torch

from prism_b200 import ops

pytestmark = pytest.mark.gpu


def _close(got, ref, what):
    g, r = got.double(), ref.double()
    rel = float((g - r).norm() / r.norm())
    mx = float((g - r).abs().max() / r.abs().max())
    assert rel <= 4e-3 and mx <= 1e-2, f"{what}: rel-L2 {rel:.2e}, max-abs/max {mx:.2e}"


def _rnd(*shape, gen, dev):
    return torch.randn(*shape, generator=gen).to(torch.bfloat16).to(dev)


@pytest.mark.parametrize("M,N,K", [(1000, 768, 512), (300, 264, 200), (128, 256, 64)])
def test_forward_dgrad_wgrad(M, N, K, cuda):
    g = torch.Generator().manual_seed(M + N + K)
    x = _rnd(M, K, gen=g, dev=cuda)
    W = _rnd(N, K, gen=g, dev=cuda)
    bias = torch.randn(N, generator=g).to(cuda)
    dy = _rnd(M, N, gen=g, dev=cuda)
    y = ops.gemm(x, W, bias=bias)
    _close(y, x.float() @ W.float().t() + bias, "forward")
    assert torch.equal(y, ops.gemm(x, W, bias=bias))
    dx = ops.gemm(dy, W, b_mn=True)                  # A = dy [M, N] K-major, B = W MN-major
    _close(dx, dy.float() @ W.float(), "dgrad")
    dW = ops.gemm(dy, x, a_mn=True, b_mn=True)       # A = dy MN-major, B = x MN-major
    _close(dW, dy.float().t() @ x.float(), "wgrad")


def test_accumulate_and_strided_output(cuda):
    g = torch.Generator().manual_seed(7)
    M, N, K = 257, 512, 384
    a1, a2 = _rnd(M, K, gen=g, dev=cuda), _rnd(M, K, gen=g, dev=cuda)
    b1, b2 = _rnd(N, K, gen=g, dev=cuda), _rnd(N, K, gen=g, dev=cuda)
    big = torch.zeros(M, N + 64, dtype=torch.bfloat16, device=cuda)
    out = big[:, 32:32 + N]
    ops.gemm(a1, b1, out=out)
    ops.gemm(a2, b2, out=out, accumulate=True)
    _close(out, a1.float() @ b1.float().t() + a2.float() @ b2.float().t(), "accumulate")
    assert not big[:, :32].any() and not big[:, 32 + N:].any()
