"""Shared tolerances and comparison helpers for the parity tests."""

import numpy as np
import torch

# Tolerances of the north-star spec: max relative error, norm-wise
# (max |y - r| / max |r| over the tensor), against an fp32-or-better reference.
TOL = {'float32': 1e-4, 'float64': 1e-10, 'bfloat16': 2e-2, 'float16': 2e-2}


def norm_rel_err(y, r) -> float:
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    if r.size == 0:
        return 0.0
    scale = float(np.max(np.abs(r)))
    return float(np.max(np.abs(y - r))) / max(scale, 1e-30)


def to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    return t.numpy() if t.dtype == torch.float64 else t.float().numpy()
