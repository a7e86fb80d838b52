"""Multi-GPU checks of the Ulysses path over NCCL (GPUs of one node; skipped when
the box has fewer than the test needs):
* tests/mp_sp_layer.py: the fused layer (uniform attention) at SP = 2 against SP = 1;
* tests/mp_sp_dynamic.py: the dynamic block-shape layer at SP = 2 and SP = 4 against
  SP = 1 (shape ids equal on every rank, outputs and gradients equal)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(script, n):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), os.path.join(HERE, script)]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)


def test_fused_layer_sp2_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    r = _run("mp_sp_layer.py", 2)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert "sp2:" in r.stdout


@pytest.mark.parametrize("n", [2, 4])
def test_dynamic_layer_sp_nccl(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    r = _run("mp_sp_dynamic.py", n)
    print(r.stdout)
    assert r.returncode == 0, (r.stdout[-3000:], r.stderr[-3000:])
    assert r.stdout.count(f"sp{n} ") == 3
