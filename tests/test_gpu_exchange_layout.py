"""The Ulysses exchange's layout changes on the GPU (prism_copy_rows) against the same
layout changes written as torch permute copies: sequence side [1, n, P*hp, D] <-> wire
[P, 1, C, hp, D], bit for bit, with a short last shard (n < C) and odd head counts."""
import pytest
import torch

from prism_b200 import _lib, communications as comm, ops

pytestmark = pytest.mark.gpu


def _torch_seq_to_wire(x, P, C, hp):
    B, n, Hp, D = x.shape
    wire = torch.zeros(P, B, C, hp, D, dtype=x.dtype, device=x.device)
    wire[:, :, :n] = x.unflatten(2, (P, hp)).permute(2, 0, 1, 3, 4)
    return wire


@pytest.mark.parametrize("P,hp,D,n,C", [(2, 20, 128, 37800, 37800), (4, 3, 128, 1001, 1003),
                                        (8, 5, 64, 777, 800), (3, 1, 16, 65, 65)])
def test_seq_wire_round_trip(P, hp, D, n, C, cuda):
    g = torch.Generator(device=cuda).manual_seed(P * 100 + hp)
    x = torch.randn(1, n, P * hp, D, generator=g, device=cuda).to(torch.bfloat16)
    wire = comm._seq_to_wire(x, P, C, hp)
    ref = _torch_seq_to_wire(x, P, C, hp)
    assert torch.equal(wire, ref)
    back = comm._wire_to_seq(wire, n)
    assert torch.equal(back, x)
    # a token-strided view (rows further apart than P*hp*D) takes the kernel path too
    big = torch.randn(1, n, P * hp + 2, D, generator=g, device=cuda).to(torch.bfloat16)
    view = big[:, :, :P * hp]
    assert torch.equal(comm._seq_to_wire(view, P, C, hp), _torch_seq_to_wire(view, P, C, hp))


def test_copy_rows_rejects_misaligned(cuda):
    a = torch.zeros(64, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.PrismError):
        ops.copy_rows(a, (0, 4), b, (0, 4), 1, 2, 4)  # 8-byte rows: refused before any launch
