"""Batched matrix products on the tcgen05 tensor cores (``avey_gemm_v1``).

``bmm(a, b)`` computes ``a @ b`` for ``a [B, m, k]`` and ``b [B, k, n]`` of
bf16 or f16 with fp32 accumulation, reading each operand through its strides:
an operand whose last dimension is contiguous is passed K-major (``a``) or
MN-major (``b``), one whose second-to-last dimension is contiguous the other
way round, so transposed views (``z.transpose(1, 2)``) cost no copy. A batch
stride of 0 (an expanded operand) shares it across the batch. ``mode`` names
the causal structure that lets tiles or K ranges be skipped (the constants
below); the result is then defined only where that structure says.

The reference has no counterpart: it multiplies with ``torch.matmul`` and
Triton's ``tl.dot`` (avey_kernels/ops.py:61-91, _triton.py:83-105). These
products serve the backward pass of the contextualizer, the enricher that
feeds it and the static layers (``layers.py``).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native

DENSE, LOWER_OUT, K_LOWER, K_UPPER = 0, 1, 2, 3
MAJOR_K, MAJOR_MN = 0, 1
KERNEL_AUTO, KERNEL_SINGLE, KERNEL_PAIR = 0, 1, 2

_DT = {torch.bfloat16: _native.AVEY_BF16, torch.float16: _native.AVEY_F16,
       torch.float32: _native.AVEY_F32}


def _layout_a(a: torch.Tensor):
    """(major, ld) of a [B, m, k] operand, or None when neither of its last two
    dimensions is contiguous."""
    if a.stride(2) == 1 and (a.shape[1] == 1 or a.stride(1) >= a.shape[2]):
        return MAJOR_K, a.stride(1) if a.shape[1] > 1 else a.shape[2]
    if a.stride(1) == 1 and (a.shape[2] == 1 or a.stride(2) >= a.shape[1]):
        return MAJOR_MN, a.stride(2) if a.shape[2] > 1 else a.shape[1]
    return None


def _layout_b(b: torch.Tensor):
    """(major, ld) of a [B, k, n] operand (K-major: k contiguous)."""
    if b.stride(1) == 1 and (b.shape[2] == 1 or b.stride(2) >= b.shape[1]):
        return MAJOR_K, b.stride(2) if b.shape[2] > 1 else b.shape[1]
    if b.stride(2) == 1 and (b.shape[1] == 1 or b.stride(1) >= b.shape[2]):
        return MAJOR_MN, b.stride(1) if b.shape[1] > 1 else b.shape[2]
    return None


def _aligned(t: torch.Tensor, *strides: int) -> bool:
    es = t.element_size()
    return t.data_ptr() % 16 == 0 and all((s * es) % 16 == 0 for s in strides)


def supported(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Whether ``bmm(a, b)`` can run natively for these operands (CUDA, bf16 /
    f16, one contiguous dimension each, 16-byte aligned bases and strides)."""
    if not (a.is_cuda and b.is_cuda) or a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float16):
        return False
    if a.dim() != 3 or b.dim() != 3 or a.shape[0] != b.shape[0] or a.shape[2] != b.shape[1]:
        return False
    la, lb = _layout_a(a), _layout_b(b)
    if la is None or lb is None:
        return False
    return _aligned(a, la[1], a.stride(0)) and _aligned(b, lb[1], b.stride(0))


def _params(a, b, c, mode, kernel=KERNEL_AUTO):
    la, lb = _layout_a(a), _layout_b(b)
    p = _native.AveyGemmParams()
    p.struct_size = ctypes.sizeof(_native.AveyGemmParams)
    p.dtype = _DT[a.dtype]
    p.out_dtype = _DT[c.dtype]
    p.mode = int(mode)
    p.batch, p.m, p.n, p.k = a.shape[0], a.shape[1], b.shape[2], a.shape[2]
    p.a, p.a_batch_stride, p.a_ld, p.a_major = a.data_ptr(), a.stride(0) if a.shape[0] > 1 else 0, la[1], la[0]
    p.b, p.b_batch_stride, p.b_ld, p.b_major = b.data_ptr(), b.stride(0) if b.shape[0] > 1 else 0, lb[1], lb[0]
    p.c, p.c_batch_stride, p.c_ld = c.data_ptr(), c.stride(0), c.stride(1) if c.shape[1] > 1 else c.shape[2]
    p.kernel = int(kernel)
    return p


def bmm(a: torch.Tensor, b: torch.Tensor, mode: int = DENSE, out: Optional[torch.Tensor] = None,
        out_dtype: torch.dtype = torch.float32, kernel: int = KERNEL_AUTO) -> torch.Tensor:
    """``a @ b`` in fp32 (or ``out_dtype`` = the operand type) on tcgen05
    (``kernel``: single-CTA tiles, CTA pairs, or AUTO = single-CTA tiles).

    Raises ``ValueError`` for operands the kernel cannot take (see
    ``supported``); there is no fallback here."""
    if not supported(a, b):
        raise ValueError('avey_gemm_v1 needs CUDA bf16 / f16 [B, m, k] and [B, k, n] operands with one '
                         'contiguous dimension each and 16-byte aligned bases and strides')
    if out is None:
        out = torch.empty(a.shape[0], a.shape[1], b.shape[2], dtype=out_dtype, device=a.device)
    p = _params(a, b, out, mode, kernel)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    with torch.cuda.device(a.device):
        _native.gemm(p, stream)
    return out
