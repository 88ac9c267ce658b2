"""Shared helpers for the parity tests."""
import numpy as np


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


# Tolerance for fp32-accumulated matvec / attention outputs against the
# reference CPU path (relative L2 <= 1e-3).
REL_L2_TOL = 1e-3


def to_dev(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def from_dev(t):
    return t.detach().cpu().numpy()
