"""Differentiable PyTorch path (``backend='torch'``).

This is the path the reference takes for autograd and CPU tensors
(avey_kernels/ops.py:94-106): plain tensor ops with fp32 accumulation (fp64
kept for gradcheck). It is not the inference hot path -- CUDA inference inputs
go to the native kernels -- and it is not the test oracle (``oracle/``).

Math per ops.py:61-91: padded rows are replaced by zeros before any
arithmetic (so NaN padding cannot reach values or gradients), rows are
L2-normalised with ``x / max(||x||, norm_eps)``, S = N N^T is weighted by V,
masked (causal keeps the diagonal; padded keys zero whole columns), mixed into
the un-normalised tail, optionally divided by the signed row sum + eps, then
bias, activation and the gate follow, and padded output rows are zero.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def activation_fn(x: torch.Tensor, activation: str) -> torch.Tensor:
    if activation == 'relu':
        return torch.relu(x)
    if activation == 'relu2':
        return torch.relu(x) ** 2
    if activation == 'silu':
        return F.silu(x)
    if activation == 'gelu':
        return F.gelu(x, approximate='tanh')
    return x


def contextualize(z_tr, v, z_tl, bias, valid, *, eps: float, norm_eps: float, causal: bool,
                  normalize: bool, activation: str) -> torch.Tensor:
    acc = torch.float64 if z_tr.dtype == torch.float64 else torch.float32
    z = z_tr.to(acc)
    zero = z.new_zeros(())
    keep_row = valid[:, :, None] if valid is not None else None
    if keep_row is not None:
        z = torch.where(keep_row, z, zero)
    norm = torch.linalg.vector_norm(z, dim=-1, keepdim=True).clamp_min(norm_eps)
    zn = z / norm
    sim = zn @ zn.transpose(-1, -2)
    if v is not None:
        sim = sim * v.to(acc)
    c = z.shape[1]
    allowed = None
    if causal:
        allowed = torch.ones(c, c, dtype=torch.bool, device=z.device).tril()[None]
    if valid is not None:
        key_ok = valid[:, None, :]
        allowed = key_ok if allowed is None else allowed & key_ok
    if allowed is not None:
        sim = torch.where(allowed, sim, zero)
    mixed = sim @ z
    if normalize:
        mixed = mixed / (sim.sum(dim=-1, keepdim=True) + eps)
    if bias is not None:
        mixed = mixed + bias.to(acc)
    y = activation_fn(mixed, activation)
    if z_tl is not None:
        gate = z_tl.to(acc)
        if keep_row is not None:
            gate = torch.where(keep_row, gate, zero)
        y = y * gate
    if keep_row is not None:
        y = torch.where(keep_row, y, zero)
    return y.to(z_tr.dtype)
