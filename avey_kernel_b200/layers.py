"""The layers on either side of the contextualizer, on the tcgen05 GEMM.

The reference leaves them to the caller ("Avey-B's static layers are
ordinary matrix multiplications and are outside this module",
avey_kernels/ops.py:1-7) and hands the contextualizer ``.contiguous()``
copies of the head and tail halves of the enriched tensor (ops.py:109-114).
Here they run on this library's batched tcgen05 matrix product
(``avey_gemm_v1``) with their elementwise work fused into its epilogue:

* ``enrich``: the enricher projection ``e = act(x W^T + b)`` into one
  ``[B, C, 2d']`` tensor whose halves ``e[..., :d']`` (head, the gate) and
  ``e[..., d':]`` (tail) feed the contextualizer as strided views, and,
  from the same epilogue, the row sums of squares of the tail half (the
  contextualizer's L2 normalisation then needs no pass over z_tr);
* ``avey_enriched`` / ``avey_b_enriched``: enricher + contextualizer, the
  second step through ``avey_fwd_presummed_v1`` (no row-norm pre-pass);
* ``static_linear``: a position-wise static layer ``act(x W^T + b) (.) gate``;
* ``static_mix``: a token-mixing static layer ``act(W z + b) (.) gate`` with a
  learned ``[C, C]`` matrix shared by the batch (lower-triangular under
  ``causal``), the static counterpart of the contextualizer's
  ``(S (.) V) z``.

CUDA inputs run natively (bf16 / f16, 16-byte aligned rows) and raise
``ValueError`` otherwise; CPU inputs take plain PyTorch, like the
contextualizer's CPU path. Inputs that require grad take PyTorch's
``F.linear`` / ``matmul`` for these layers (with autograd) and the native
contextualizer and its native backward.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import _native, gemm, ops

_ACT_IDS = _native.ACTIVATION_IDS
_DT = {torch.bfloat16: _native.AVEY_BF16, torch.float16: _native.AVEY_F16}


def _act_torch(y: torch.Tensor, activation: str) -> torch.Tensor:
    if activation == 'identity':
        return y
    if activation == 'relu':
        return torch.relu(y)
    if activation == 'relu2':
        return torch.relu(y).square()
    if activation == 'silu':
        return F.silu(y)
    return F.gelu(y, approximate='tanh')


def _check_act(activation: str) -> None:
    if activation not in _ACT_IDS:
        raise ValueError('unsupported activation')


def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


def _native_ok(*ts) -> bool:
    return all(t is None or (t.is_cuda and t.dtype in _DT) for t in ts)


def _epilogue_gemm(a, b, out, *, bias=None, gate=None, activation='identity', mode=gemm.DENSE,
                   sumsq=None, sumsq_col0=0):
    """One avey_gemm_v1 call with a 16-bit output and the fused epilogue."""
    if not gemm.supported(a, b):
        raise ValueError('the native layer needs bf16 / f16 CUDA operands with one contiguous '
                         'dimension and 16-byte aligned rows (feature counts multiples of 8)')
    p = gemm._params(a, b, out, mode)
    if bias is not None:
        p.bias = bias.contiguous().data_ptr()
    if gate is not None:
        if gate.stride(-1) != 1 or (gate.stride(1) * gate.element_size()) % 16 or gate.data_ptr() % 16:
            gate = gate.contiguous()
        p.gate = gate.data_ptr()
        p.gate_batch_stride = gate.stride(0) if gate.shape[0] > 1 else 0
        p.gate_ld = gate.stride(1)
    p.activation = _ACT_IDS[activation]
    if sumsq is not None:
        p.sumsq, p.sumsq_col0 = sumsq.data_ptr(), int(sumsq_col0)
    keep = (bias, gate)  # alive until the launch is enqueued
    with torch.cuda.device(a.device):
        _native.gemm(p, torch.cuda.current_stream(a.device).cuda_stream)
    del keep
    return out


def enrich(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
           activation: str = 'identity', tail_sums: bool = False
           ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Enricher projection ``e = act(x W^T + bias)``.

    x ``[B, C, d_in]``, weight ``[2d', d_in]`` (``nn.Linear`` layout), bias
    ``[2d']``. Returns ``(e, sums)``: e ``[B, C, 2d']`` in x's dtype, and with
    ``tail_sums`` (native path, d' a multiple of 128) the row sums of squares
    of ``e[..., d':]`` as ``[d' / 128, B * C]`` fp32 planes (else None)."""
    _check_act(activation)
    if x.ndim != 3 or weight.ndim != 2 or weight.shape[1] != x.shape[2] or weight.shape[0] % 2:
        raise ValueError('x must be [batch, context, d_in] and weight [2 d\', d_in]')
    if bias is not None and tuple(bias.shape) != (weight.shape[0],):
        raise ValueError('bias must have shape [2 d\']')
    if not x.is_cuda or _needs_grad(x, weight, bias):
        return _act_torch(F.linear(x, weight, bias), activation), None
    if not _native_ok(x, weight, bias) or weight.dtype != x.dtype or (bias is not None and bias.dtype != x.dtype):
        raise ValueError('the native enricher takes bf16 / f16 CUDA tensors of one dtype')
    bt, c, _ = x.shape
    n = weight.shape[0]
    d = n // 2
    out = torch.empty(bt, c, n, dtype=x.dtype, device=x.device)
    sums = None
    if tail_sums and d % 128 == 0:
        sums = torch.empty(d // 128, bt * c, dtype=torch.float32, device=x.device)
    xa = x if x.stride(-1) == 1 else x.contiguous()
    wt = weight.t().unsqueeze(0).expand(bt, weight.shape[1], n)  # [B, d_in, 2d'], K-major
    _epilogue_gemm(xa, wt, out, bias=bias, activation=activation, sumsq=sums, sumsq_col0=d)
    return out, sums


def _contextualize_presummed(z_tr, v, z_tl, bias, valid, sums, *, eps, norm_eps, causal,
                             normalize, activation):
    """The native contextualizer with the row sums of squares of z_tr given
    (``avey_fwd_presummed_v1``)."""
    out = torch.empty(z_tr.shape, dtype=z_tr.dtype, device=z_tr.device)
    params = ops.build_params(z_tr, v, z_tl, bias, valid, out, eps=eps, norm_eps=norm_eps,
                              causal=causal, normalize=normalize,
                              activation_id=_ACT_IDS[activation])
    # Up to 512 tokens the planes are combined into a workspace of one float
    # per row; above, the long-context path's workspace.
    nbytes = max(_native.workspace_size(params), 4 * z_tr.shape[0] * z_tr.shape[1])
    with torch.cuda.device(z_tr.device):
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=z_tr.device)
        params.workspace, params.workspace_bytes = ws.data_ptr(), nbytes
        _native.forward_presummed(params, sums.data_ptr(), sums.shape[0],
                                  torch.cuda.current_stream(z_tr.device).cuda_stream)
    return out


def _enriched(x, enrich_weight, v, enrich_bias, enrich_activation, bias, valid, eps, norm_eps,
              causal, normalize, activation):
    e, sums = enrich(x, enrich_weight, enrich_bias, activation=enrich_activation,
                     tail_sums=True)
    d = e.shape[-1] // 2
    head, tail = e[..., :d], e[..., d:]
    if sums is None or not e.is_cuda or _needs_grad(e, v, bias):
        if normalize:
            return ops.avey_b(tail, z_tl=head, bias=bias, valid=valid, eps=eps, norm_eps=norm_eps,
                              activation=activation)
        return ops.avey(tail, v, z_tl=head, bias=bias, valid=valid, causal=causal,
                        norm_eps=norm_eps, activation=activation)
    ops._validate(tail, v, head, bias, valid, eps, norm_eps, activation, 'cuda', 32, False)
    return _contextualize_presummed(tail, v, head, bias, valid, sums, eps=eps, norm_eps=norm_eps,
                                    causal=causal, normalize=normalize, activation=activation)


def avey_enriched(x: torch.Tensor, enrich_weight: torch.Tensor, v: torch.Tensor, *,
                  enrich_bias=None, enrich_activation='identity', bias=None, valid=None,
                  causal=True, norm_eps=1e-12, activation='identity') -> torch.Tensor:
    """Enricher then Avey contextualizer: ``avey(e[..., d':], v, z_tl=e[...,
    :d'], ...)`` with ``e = enrich(x, enrich_weight, enrich_bias)``, the
    contextualizer taking the tail's row norms from the enricher's epilogue."""
    return _enriched(x, enrich_weight, v, enrich_bias, enrich_activation, bias, valid, 1e-6,
                     norm_eps, causal, False, activation)


def avey_b_enriched(x: torch.Tensor, enrich_weight: torch.Tensor, *, enrich_bias=None,
                    enrich_activation='identity', bias=None, valid=None, eps=1e-6,
                    norm_eps=1e-12, activation='identity') -> torch.Tensor:
    """Enricher then Avey-B contextualizer (see ``avey_enriched``)."""
    return _enriched(x, enrich_weight, None, enrich_bias, enrich_activation, bias, valid, eps,
                     norm_eps, False, True, activation)


def static_linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
                  activation: str = 'identity', gate: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Position-wise static layer ``act(x W^T + bias) (.) gate``: x ``[B, C,
    d_in]``, weight ``[d_out, d_in]``, bias ``[d_out]``, gate ``[B, C, d_out]``."""
    _check_act(activation)
    if x.ndim != 3 or weight.ndim != 2 or weight.shape[1] != x.shape[2]:
        raise ValueError('x must be [batch, context, d_in] and weight [d_out, d_in]')
    d_out = weight.shape[0]
    if bias is not None and tuple(bias.shape) != (d_out,):
        raise ValueError('bias must have shape [d_out]')
    if gate is not None and tuple(gate.shape) != (*x.shape[:2], d_out):
        raise ValueError('gate must have shape [batch, context, d_out]')
    if not x.is_cuda or _needs_grad(x, weight, bias, gate):
        y = _act_torch(F.linear(x, weight, bias), activation)
        return y * gate if gate is not None else y
    if not _native_ok(x, weight, bias, gate) or any(t is not None and t.dtype != x.dtype
                                                    for t in (weight, bias, gate)):
        raise ValueError('the native static layer takes bf16 / f16 CUDA tensors of one dtype')
    bt, c, d_in = x.shape
    out = torch.empty(bt, c, d_out, dtype=x.dtype, device=x.device)
    xa = x if x.stride(-1) == 1 else x.contiguous()
    wt = weight.t().unsqueeze(0).expand(bt, d_in, d_out)
    return _epilogue_gemm(xa, wt, out, bias=bias, gate=gate, activation=activation)


def static_mix(z: torch.Tensor, weight: torch.Tensor, *, bias: Optional[torch.Tensor] = None,
               activation: str = 'identity', gate: Optional[torch.Tensor] = None,
               causal: bool = False) -> torch.Tensor:
    """Token-mixing static layer ``act(W z[b] + bias) (.) gate[b]`` for every
    batch row: z ``[B, C, d]``, weight ``[C, C]`` indexed [query, key] (only its
    lower triangle, diagonal kept, under ``causal``), bias ``[d]``, gate
    ``[B, C, d]``."""
    _check_act(activation)
    if z.ndim != 3 or tuple(weight.shape) != (z.shape[1], z.shape[1]):
        raise ValueError('z must be [batch, context, d] and weight [context, context]')
    if bias is not None and tuple(bias.shape) != (z.shape[2],):
        raise ValueError('bias must have shape [d]')
    if gate is not None and tuple(gate.shape) != tuple(z.shape):
        raise ValueError('gate must have the shape of z')
    w = weight.tril() if causal else weight
    if not z.is_cuda or _needs_grad(z, weight, bias, gate):
        y = torch.matmul(w, z)
        if bias is not None:
            y = y + bias
        y = _act_torch(y, activation)
        return y * gate if gate is not None else y
    if not _native_ok(z, weight, bias, gate) or any(t is not None and t.dtype != z.dtype
                                                    for t in (weight, bias, gate)):
        raise ValueError('the native static layer takes bf16 / f16 CUDA tensors of one dtype')
    bt, c, d = z.shape
    out = torch.empty(bt, c, d, dtype=z.dtype, device=z.device)
    wa = (w if w.stride(-1) == 1 else w.contiguous()).unsqueeze(0).expand(bt, c, c)
    za = z if z.stride(-1) == 1 else z.contiguous()
    return _epilogue_gemm(wa, za, out, bias=bias, gate=gate, activation=activation,
                          mode=gemm.K_LOWER if causal else gemm.DENSE)
