"""CPU oracle for the contextualizer's gradients.

TEST INFRASTRUCTURE ONLY, like ``contextualizer.py``: the checker for the
native backward (``avey_kernel_b200/backward.py``), never called by it.

The reference has no hand-written backward: its gradients are torch autograd
through ``avey_kernels/ops.py::_reference`` (ops.py:61-91; the reference's
tests/test_contextualizer.py:41-62 gradcheck it and check NaN padding). This
module restates that chain rule in NumPy, step by step against the forward
lines it differentiates:

* ops.py:89-91   rows of padded queries get no gradient (masked_fill).
* ops.py:84-88   d gate = dout * act(Ypre); dA = dout * gate (padded rows 0).
* ops.py:81-83   dYpre = dA * act'(Ypre) with torch's derivative conventions
                 (relu' = [x > 0], relu2' = 2 max(x, 0), silu' = s (1 + x (1 - s)),
                 tanh-gelu' = 0.5 (1 + t) + 0.5 x (1 - t^2) k (1 + 3 c x^2));
                 d bias = sum over rows of dYpre.
* ops.py:79-80   Avey-B: dnum = dYpre / den, dden_i = -sum_f dYpre_if Y0_if / den_i.
* ops.py:78      dS = dnum Z^T (+ dden along the row), dZ += S^T dnum.
* ops.py:69-77   masked entries of S pass no gradient; dV = sum_b dS (.) G,
                 dG = dS (.) V, dZhat = (dG + dG^T) Zhat.
* ops.py:68      F.normalize: dZ += (dZhat - Zhat (Zhat . dZhat)) / ||Z|| where
                 ||Z|| >= norm_eps, dZhat / norm_eps below (clamp_min passes no
                 gradient to the norm there).
* ops.py:64-67   padded rows of z_tr get no gradient (masked_fill before use).

Pinned by ``tests/test_oracle_backward.py`` against gradients of the reference
itself (``tests/golden/make_grad_golden.py``) and against finite differences.
"""

from __future__ import annotations

import math

import numpy as np

from .contextualizer import _sigmoid, activate


def activate_grad(x: np.ndarray, activation: str) -> np.ndarray:
    """Derivative of ``activate`` at x (torch's autograd conventions)."""
    if activation == 'identity':
        return np.ones_like(x)
    if activation == 'relu':
        return (x > 0).astype(x.dtype)
    if activation == 'relu2':
        return np.where(x > 0, 2 * x, 0).astype(x.dtype)
    if activation == 'silu':
        with np.errstate(over='ignore'):
            s = _sigmoid(x)
        return s * (1 + x * (1 - s))
    if activation == 'gelu':
        k, c = math.sqrt(2.0 / math.pi), 0.044715
        t = np.tanh(k * (x + c * x * x * x))
        return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * k * (1 + 3 * c * x * x)
    raise ValueError(f'unsupported activation {activation!r}')


def contextualize_backward(z_tr, v=None, z_tl=None, bias=None, valid=None, grad_out=None, *,
                           eps: float, norm_eps: float, causal: bool, normalize: bool,
                           activation: str = 'identity', accum=np.float64):
    """Gradients (z_tr, v, z_tl, bias) of ``contextualize`` for the upstream
    gradient ``grad_out``; absent inputs get None. Arrays are ``accum``."""
    z = np.asarray(z_tr, dtype=accum)
    b, c, d = z.shape
    ok = np.ones((b, c), dtype=bool) if valid is None else np.asarray(valid, dtype=bool)
    zm = np.where(ok[:, :, None], z, 0)
    norm = np.sqrt(np.einsum('bcd,bcd->bc', zm, zm))
    nrm = np.maximum(norm, norm_eps)
    zh = zm / nrm[:, :, None]
    g = zh @ np.swapaxes(zh, 1, 2)
    allowed = np.broadcast_to(ok[:, None, :], (b, c, c))
    if causal:
        allowed = allowed & np.tril(np.ones((c, c), dtype=bool))[None]
    vv = np.ones((c, c), dtype=accum) if v is None else np.asarray(v, dtype=accum)
    s = np.where(allowed, g * vv[None], 0)
    num = s @ zm
    den = s.sum(axis=-1) + accum(eps)
    y0 = num / den[:, :, None] if normalize else num
    ypre = y0 + (0 if bias is None else np.asarray(bias, dtype=accum))
    go = np.where(ok[:, :, None], np.asarray(grad_out, dtype=accum), 0)
    gate = None
    d_gate = None
    if z_tl is not None:
        gate = np.where(ok[:, :, None], np.asarray(z_tl, dtype=accum), 0)
        d_gate = np.where(ok[:, :, None], go * activate(ypre, activation), 0)
    da = go if gate is None else go * gate
    dy = np.where(ok[:, :, None], da * activate_grad(ypre, activation), 0)
    d_bias = None if bias is None else dy.sum(axis=(0, 1))
    if normalize:
        dnum = dy / den[:, :, None]
        dden = -(dy * y0).sum(axis=-1) / den
    else:
        dnum = dy
        dden = np.zeros((b, c), dtype=accum)
    ds = np.where(allowed, dnum @ np.swapaxes(zm, 1, 2) + dden[:, :, None], 0)
    d_v = None if v is None else (ds * g).sum(axis=0)
    dg = ds * vv[None]
    dzh = (dg + np.swapaxes(dg, 1, 2)) @ zh
    dot = np.einsum('bcd,bcd->bc', zh, dzh)
    scaled = (norm >= norm_eps)[:, :, None]
    dz_norm = np.where(scaled, (dzh - zh * dot[:, :, None]) / nrm[:, :, None], dzh / norm_eps)
    d_z = np.where(ok[:, :, None], dz_norm + np.swapaxes(s, 1, 2) @ dnum, 0)
    return d_z, d_v, d_gate, d_bias
