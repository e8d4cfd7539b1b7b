"""CPU oracle for the Avey / Avey-B contextualizer forward pass.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA path is
compared against; it is never called by the product path (``avey_kernel_b200``),
which raises when its CUDA library is missing instead of falling back here.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.

It restates, in NumPy, the reference implementation
``avey_kernels/ops.py::_reference`` (HusamettinYilmazz/avey_kernel), step by
step; the line numbers below are those of that file:

* ops.py:63      accumulate in fp32 (fp64 kept for fp64 input).  The oracle
                 accumulates in ``accum`` (fp64 by default: a tighter truth
                 than the reference's own fp32 arithmetic).
* ops.py:64-67   zero invalid rows *before* any arithmetic (NaN padding).
* ops.py:68      ``F.normalize(x, p=2, dim=-1, eps)`` = x / max(||x||, eps).
* ops.py:69      cosine similarity S = N N^T.
* ops.py:70-71   S *= V (Avey only), V indexed [query, key].
* ops.py:72-75   causal mask keeps j <= i (the diagonal is kept).
* ops.py:76-77   invalid keys zero whole columns of S.
* ops.py:78      numerator = S @ z_tr (the *un-normalised* tail).
* ops.py:79-80   Avey-B: divide by the signed row sum plus eps.
* ops.py:81-83   + bias, then the activation (ops.py:49-58).
* ops.py:84-88   multiply by the gate z_tl with invalid rows zeroed.
* ops.py:89-91   zero invalid output rows; cast back to the input dtype
                 (the caller does the cast: the oracle returns ``accum``).

Parity pin: ``tests/test_oracle.py`` checks this oracle against the
hand-computed fixtures of the reference's own tests
(tests/test_contextualizer.py:13-39, tests/test_profiling.py:46-61,
tests/test_triton.py:162-169) and against golden vectors produced by running
the reference's ``_reference`` (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math

import numpy as np

ACTIVATIONS = ('identity', 'relu', 'relu2', 'silu', 'gelu')


def activate(x: np.ndarray, activation: str) -> np.ndarray:
    """ops.py:49-58: identity, relu, relu^2, silu and tanh-approximate gelu."""
    if activation == 'identity':
        return x
    if activation == 'relu':
        return np.maximum(x, 0)
    if activation == 'relu2':
        r = np.maximum(x, 0)
        return r * r
    if activation == 'silu':
        # x * sigmoid(x), written so that large |x| neither overflows nor NaNs.
        with np.errstate(over='ignore'):
            return x * _sigmoid(x)
    if activation == 'gelu':
        # PyTorch's approximate='tanh': 0.5 x (1 + tanh(sqrt(2/pi)(x + 0.044715 x^3))).
        inner = math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)
        return 0.5 * x * (1.0 + np.tanh(inner))
    raise ValueError(f'unsupported activation {activation!r}')


def _sigmoid(x: np.ndarray) -> np.ndarray:
    e = np.exp(-np.abs(x))
    return np.where(x >= 0, 1.0 / (1.0 + e), e / (1.0 + e))


def contextualize(z_tr, v=None, z_tl=None, bias=None, valid=None, *,
                  eps: float, norm_eps: float, causal: bool, normalize: bool,
                  activation: str = 'identity', accum=np.float64) -> np.ndarray:
    """Contextualizer forward for every batch row; returns an ``accum`` array.

    Shapes: z_tr, z_tl [B, C, d]; v [C, C]; bias [d]; valid [B, C] bool.
    """
    z = np.asarray(z_tr, dtype=accum)
    if z.ndim != 3:
        raise ValueError('z_tr must be [batch, context, features]')
    b, c, _ = z.shape
    row_ok = None
    if valid is not None:
        row_ok = np.asarray(valid, dtype=bool)
        z = np.where(row_ok[:, :, None], z, 0)
    norms = np.sqrt(np.einsum('bcd,bcd->bc', z, z))
    zn = z / np.maximum(norms, norm_eps)[:, :, None]
    s = zn @ np.swapaxes(zn, 1, 2)
    if v is not None:
        s = s * np.asarray(v, dtype=accum)[None]
    if causal:
        s = np.where(np.tril(np.ones((c, c), dtype=bool))[None], s, 0)
    if row_ok is not None:
        s = np.where(row_ok[:, None, :], s, 0)
    num = s @ z
    if normalize:
        num = num / (s.sum(axis=-1, keepdims=True) + accum(eps))
    if bias is not None:
        num = num + np.asarray(bias, dtype=accum)
    out = activate(num, activation)
    if z_tl is not None:
        gate = np.asarray(z_tl, dtype=accum)
        if row_ok is not None:
            gate = np.where(row_ok[:, :, None], gate, 0)
        out = out * gate
    if row_ok is not None:
        out = np.where(row_ok[:, :, None], out, 0)
    return out


def avey(z_tr, v, *, z_tl=None, bias=None, valid=None, causal=True,
         norm_eps=1e-12, activation='identity', accum=np.float64):
    """ops.py:117-133: Avey (learned V, eps fixed at 1e-6, no row-sum divide)."""
    if v is None:
        raise ValueError('Avey requires the learned V matrix (v)')
    return contextualize(z_tr, v, z_tl, bias, valid, eps=1e-6, norm_eps=norm_eps,
                         causal=causal, normalize=False, activation=activation,
                         accum=accum)


def avey_b(z_tr, *, z_tl=None, bias=None, valid=None, eps=1e-6, norm_eps=1e-12,
           activation='identity', accum=np.float64):
    """ops.py:136-147: Avey-B (no V, bidirectional, signed row-sum divide)."""
    return contextualize(z_tr, None, z_tl, bias, valid, eps=eps, norm_eps=norm_eps,
                         causal=False, normalize=True, activation=activation,
                         accum=accum)


def allowed_pairs(c: int, causal: bool, valid=None) -> np.ndarray:
    """Number of (query, key) pairs that contribute per batch row.

    Used for the algorithmic FLOP count: a pair costs 2d for S and 2d for the
    mix. Causal keeps j <= i; a padding mask keeps valid query and key rows.
    """
    if valid is None:
        per = c * (c + 1) // 2 if causal else c * c
        return np.full(1, per, dtype=np.int64)
    ok = np.asarray(valid, dtype=bool)
    if not causal:
        n = ok.sum(axis=1).astype(np.int64)
        return n * n
    # causal with holes: for each valid query i count valid keys j <= i
    cum = np.cumsum(ok, axis=1)
    return (cum * ok).sum(axis=1).astype(np.int64)
