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
