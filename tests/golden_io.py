"""Load golden fixtures and rebuild their seeded inputs (shared by CPU and GPU tests)."""

import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def np32(t):
    """torch tensor (any float dtype, CPU) -> float32 numpy array holding the same values."""
    return t.detach().float().cpu().numpy()
