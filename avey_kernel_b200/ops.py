"""Public operations: drop-in for ``avey_kernels.ops`` (``avey``, ``avey_b``).

Same signatures, tensor conventions and errors as the reference
(avey_kernels/ops.py:23-147). Backends:

* ``'cuda'``  the native sm_100a kernels through the C ABI (``libavey_b200.so``)
  for CUDA tensors, otherwise ``ValueError``. Inputs that require grad get the
  native backward (``backward.py``); the reference has none and sends them to
  its PyTorch path (ops.py:94-106).
* ``'triton'`` accepted for source compatibility: it names the fused GPU
  kernel, which here is the native CUDA one, under the reference's rules for
  that backend (ops.py:98-103): CUDA fp16 / bf16 / fp32 inference inputs only,
  so fp64 inputs, CPU tensors and inputs that require grad raise
  ``ValueError`` as they do in the reference.
* ``'torch'`` the differentiable PyTorch path (``eager.py``).
* ``'auto'``  ``'cuda'`` for CUDA tensors, with or without autograd; the
  PyTorch path for CPU tensors.

The native path never falls back silently: when the library is missing or the
device is not sm_100, the call raises.

``output_tile`` and ``autotune`` are validated like the reference does and
otherwise ignored: the CUDA kernels pick their tiling from the shape.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch

from . import _native, backward, eager

_BACKENDS = ('auto', 'torch', 'cuda', 'triton')
_ACTIVATIONS = tuple(_native.ACTIVATION_IDS)
_DTYPE_IDS = {torch.float32: _native.AVEY_F32, torch.float16: _native.AVEY_F16,
              torch.bfloat16: _native.AVEY_BF16, torch.float64: _native.AVEY_F64}


def _validate(z_tr, v, z_tl, bias, valid, eps, norm_eps, activation, backend, output_tile,
              autotune):
    """Input contract of the reference (ops.py:23-46); violations raise ValueError."""
    if not isinstance(z_tr, torch.Tensor) or z_tr.ndim != 3 or 0 in z_tr.shape:
        raise ValueError('z_tr must have nonempty shape [batch, context, features]')
    if z_tr.dtype not in _DTYPE_IDS:
        raise ValueError('z_tr must be floating point')
    if backend not in _BACKENDS:
        raise ValueError('backend must be auto, torch, cuda, or triton')
    if type(output_tile) is not int or output_tile not in (32, 64, 128):
        raise ValueError('output_tile must be 32, 64, or 128')
    if type(autotune) is not bool:
        raise ValueError('autotune must be boolean')
    if activation not in _ACTIVATIONS:
        raise ValueError('unsupported activation')
    for value in (eps, norm_eps):
        if not isinstance(value, (int, float)) or not math.isfinite(value) or value <= 0:
            raise ValueError('eps and norm_eps must be finite and positive')
    c, d_prime = z_tr.shape[1:]
    expected = {'v': (c, c), 'z_tl': tuple(z_tr.shape), 'bias': (d_prime,)}
    for name, tensor in (('v', v), ('z_tl', z_tl), ('bias', bias)):
        if tensor is None:
            continue
        if (tuple(tensor.shape) != expected[name] or tensor.device != z_tr.device
                or tensor.dtype != z_tr.dtype):
            raise ValueError(f'{name} must have shape {expected[name]}, z_tr.dtype, and z_tr.device')
    if valid is not None and (tuple(valid.shape) != tuple(z_tr.shape[:2])
                              or valid.dtype != torch.bool or valid.device != z_tr.device):
        raise ValueError('valid must be boolean [batch, context] on z_tr.device')


def _feature_major(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """The C ABI wants unit stride along the last dimension; other strides are free."""
    if t is None or t.stride(-1) == 1:
        return t
    return t.contiguous()


def _row_strides(t: torch.Tensor):
    return (t.stride(0) if t.shape[0] > 1 else t.shape[1] * t.stride(1)), t.stride(1)


def build_params(z_tr, v, z_tl, bias, valid, out, *, eps, norm_eps, causal, normalize,
                 activation_id, kernel=_native.KERNEL_AUTO) -> _native.AveyFwdParams:
    """Fill the C-ABI parameter block from tensors (pointers, element strides)."""
    p = _native.new_params()
    p.dtype = _DTYPE_IDS[z_tr.dtype]
    p.batch, p.context, p.features = (int(s) for s in z_tr.shape)
    p.z_tr = z_tr.data_ptr()
    p.z_tr_batch_stride, p.z_tr_row_stride = _row_strides(z_tr)
    if v is not None:
        p.v = v.data_ptr()
        p.v_row_stride = v.stride(0) if v.shape[0] > 1 else v.shape[1]
    if z_tl is not None:
        p.z_tl = z_tl.data_ptr()
        p.z_tl_batch_stride, p.z_tl_row_stride = _row_strides(z_tl)
    if bias is not None:
        p.bias = bias.data_ptr()
    if valid is not None:
        p.valid = valid.data_ptr()
        p.valid_batch_stride = valid.stride(0)
        p.valid_row_stride = valid.stride(1)
    p.out = out.data_ptr()
    p.out_batch_stride, p.out_row_stride = _row_strides(out)
    p.eps = float(eps)
    p.norm_eps = float(norm_eps)
    p.causal = int(bool(causal))
    p.normalize = int(bool(normalize))
    p.activation = int(activation_id)
    p.kernel = int(kernel)
    return p


def _prepare(z_tr, v, z_tl, bias, valid):
    z_tr = _feature_major(z_tr)
    z_tl = _feature_major(z_tl)
    if v is not None and v.stride(1) != 1:
        v = v.contiguous()
    if bias is not None and bias.stride(0) != 1:
        bias = bias.contiguous()
    return z_tr, v, z_tl, bias, valid


@torch.library.custom_op('avey_b200::contextualize', mutates_args=())
def contextualize(z_tr: torch.Tensor, v: Optional[torch.Tensor], z_tl: Optional[torch.Tensor],
                  bias: Optional[torch.Tensor], valid: Optional[torch.Tensor], eps: float,
                  norm_eps: float, causal: bool, normalize: bool, activation: int,
                  variant: int = 0) -> torch.Tensor:
    """Native contextualizer forward: one launch of the sm_100a library on the
    current stream. Replaces the reference's ``avey_kernels::mix`` custom op
    (_triton.py:153-188) plus its normalisation pre-pass (ops.py:107-108).
    ``variant`` selects the kernel (0 auto, 1 CUDA-core, 2 tcgen05)."""
    if not z_tr.is_cuda:
        raise ValueError('avey_b200::contextualize needs CUDA tensors')
    z_tr, v, z_tl, bias, valid = _prepare(z_tr, v, z_tl, bias, valid)
    out = torch.empty(z_tr.shape, dtype=z_tr.dtype, device=z_tr.device)
    params = build_params(z_tr, v, z_tl, bias, valid, out, eps=eps, norm_eps=norm_eps,
                          causal=causal, normalize=normalize, activation_id=activation,
                          kernel=variant)
    nbytes = _native.workspace_size(params)
    batch = z_tr.shape[0]
    # The workspace grows linearly with the batch (above 512 tokens it holds
    # P, 2 bytes per (query, key) pair); past the cap, batch slices run one
    # after the other on one workspace, so memory stays bounded.
    per_row = -(-nbytes // batch) if nbytes else 0
    step = batch if nbytes <= _workspace_cap() else max(1, _workspace_cap() // max(per_row, 1))
    stream = torch.cuda.current_stream(z_tr.device).cuda_stream
    workspace = None
    with torch.cuda.device(z_tr.device):
        for b0 in range(0, batch, step):
            b1 = min(batch, b0 + step)
            if step != batch:
                sl = slice(b0, b1)
                params = build_params(z_tr[sl], v, z_tl[sl] if z_tl is not None else None, bias,
                                      valid[sl] if valid is not None else None, out[sl], eps=eps,
                                      norm_eps=norm_eps, causal=causal, normalize=normalize,
                                      activation_id=activation, kernel=variant)
                nbytes = _native.workspace_size(params)
            if nbytes:
                if workspace is None or workspace.numel() < nbytes:
                    # Scratch from torch's caching allocator (stream-ordered, graph-safe).
                    workspace = torch.empty(nbytes, dtype=torch.uint8, device=z_tr.device)
                params.workspace = workspace.data_ptr()
                params.workspace_bytes = nbytes
            _native.forward(params, stream)
    return out


def _workspace_cap() -> int:
    """Largest workspace one launch sequence may use (bytes); the
    AVEY_B200_MAX_WORKSPACE_MB environment variable overrides 2048 MB."""
    return int(os.environ.get('AVEY_B200_MAX_WORKSPACE_MB', '2048')) << 20


@contextualize.register_fake
def _contextualize_fake(z_tr, v, z_tl, bias, valid, eps, norm_eps, causal, normalize,
                        activation, variant=0):
    return torch.empty(z_tr.shape, dtype=z_tr.dtype, device=z_tr.device)


backward.register()


@torch.library.custom_op('avey_b200::contextualize_packed', mutates_args=())
def contextualize_packed(x: torch.Tensor, v: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                         valid: Optional[torch.Tensor], eps: float, norm_eps: float, causal: bool,
                         normalize: bool, activation: int) -> torch.Tensor:
    """``contextualize`` with z_tl = x[..., :d'] and z_tr = x[..., d':] of one
    [B, C, 2d'] tensor: the same forward, one gradient for x in the backward."""
    d = x.shape[-1] // 2
    return contextualize(x[..., d:], v, x[..., :d], bias, valid, eps, norm_eps, causal, normalize,
                         activation)


@contextualize_packed.register_fake
def _contextualize_packed_fake(x, v, bias, valid, eps, norm_eps, causal, normalize, activation):
    return x.new_empty((*x.shape[:-1], x.shape[-1] // 2))


backward.register_packed()


def _packed_base(z_tr, z_tl):
    """x when z_tl is x[..., :d'] and z_tr is x[..., d':] of one [B, C, 2d']
    tensor x that requires grad (unit stride along features), else None."""
    if z_tl is None or not (z_tr.requires_grad and z_tl.requires_grad):
        return None
    try:
        base = z_tr._base
        if base is None or z_tl._base is not base or not base.requires_grad or base.dim() != 3:
            return None
        b, c, d = z_tr.shape
        if tuple(base.shape) != (b, c, 2 * d) or base.stride(-1) != 1:
            return None
        if z_tr.stride() != base.stride() or z_tl.stride() != base.stride():
            return None
        p0 = base.data_ptr()
        if z_tl.data_ptr() != p0 or z_tr.data_ptr() != p0 + d * base.element_size():
            return None
        return base
    except (AttributeError, RuntimeError):
        return None


def plan(z_tr, v=None, z_tl=None, bias=None, valid=None, *, causal=True, normalize=False,
         eps=1e-6, norm_eps=1e-12, activation='identity', kernel=_native.KERNEL_AUTO):
    """The launch the native op would make for these tensors (no launch)."""
    z_tr, v, z_tl, bias, valid = _prepare(z_tr, v, z_tl, bias, valid)
    out = torch.empty(z_tr.shape, dtype=z_tr.dtype, device=z_tr.device)
    params = build_params(z_tr, v, z_tl, bias, valid, out, eps=eps, norm_eps=norm_eps,
                          causal=causal, normalize=normalize,
                          activation_id=_native.ACTIVATION_IDS[activation], kernel=kernel)
    return _native.plan(params)


def _dispatch(z_tr, v, z_tl, bias, valid, eps, norm_eps, causal, normalize, activation, backend,
              output_tile, autotune):
    _validate(z_tr, v, z_tl, bias, valid, eps, norm_eps, activation, backend, output_tile,
              autotune)
    native_ok = z_tr.is_cuda and torch.version.hip is None
    if backend == 'triton':
        # The reference's conditions for its fused-kernel backend (ops.py:96-103).
        needs_grad = torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (z_tr, v, z_tl, bias))
        if not native_ok or z_tr.dtype == torch.float64 or needs_grad:
            raise ValueError('Triton requires Triton installed, NVIDIA SM80+, and CUDA '
                             'FP16/BF16/FP32 inference inputs; use backend="torch" for autograd')
    if backend == 'cuda' and not native_ok:
        raise ValueError('the CUDA backend needs CUDA tensors; use backend="torch" for CPU tensors')
    if backend == 'torch' or not native_ok:
        return eager.contextualize(z_tr, v, z_tl, bias, valid, eps=eps, norm_eps=norm_eps,
                                   causal=causal, normalize=normalize, activation=activation)
    if torch.is_grad_enabled():
        base = _packed_base(z_tr, z_tl)
        if base is not None:
            return contextualize_packed(base, v, bias, valid, float(eps), float(norm_eps),
                                        bool(causal), bool(normalize),
                                        _native.ACTIVATION_IDS[activation])
    return contextualize(z_tr, v, z_tl, bias, valid, float(eps), float(norm_eps), bool(causal),
                         bool(normalize), _native.ACTIVATION_IDS[activation])


def avey(z_tr: torch.Tensor, v: torch.Tensor, *, z_tl=None, bias=None, valid=None, causal=True,
         norm_eps=1e-12, activation='identity', backend='auto', output_tile=32, autotune=False):
    """Avey contextualizer: z_tl * activation(((v * cosine(z_tr, z_tr)) masked) @ z_tr + bias).

    Causal masking keeps the diagonal. ``valid`` masks both query and key
    positions; invalid output rows are zero, including after bias and gating.
    ``bias`` has shape [features]; ``z_tl``, if present, has the shape of z_tr.
    Mirrors avey_kernels/ops.py:117-133.
    """
    if v is None:
        raise ValueError('Avey requires the learned V matrix (v)')
    return _dispatch(z_tr, v, z_tl, bias, valid, 1e-6, norm_eps, causal, False, activation,
                     backend, output_tile, autotune)


def avey_b(z_tr: torch.Tensor, *, z_tl=None, bias=None, valid=None, eps=1e-6, norm_eps=1e-12,
           activation='identity', backend='auto', output_tile=32, autotune=False):
    """Avey-B dynamic mixing: z_tl * activation((S @ z_tr) / (sum(S) + eps) + bias).

    S is the cosine similarity with invalid keys zeroed; signed similarities are
    kept and the denominator is neither clamped nor a softmax. GELU uses the
    tanh approximation. Mirrors avey_kernels/ops.py:136-147.
    """
    return _dispatch(z_tr, None, z_tl, bias, valid, eps, norm_eps, False, True, activation,
                     backend, output_tile, autotune)
