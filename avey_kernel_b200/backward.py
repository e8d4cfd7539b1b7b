"""Backward of the contextualizer on the GPU, and its autograd registration.

The reference differentiates only through its PyTorch path
(avey_kernels/ops.py:94-106 route inputs that require grad to _reference,
ops.py:61-91). Here ``avey_b200::contextualize`` (the native forward) gets a
native backward: five batched GEMMs (this library's tcgen05 kernel,
``avey_gemm_v1``, for bf16 inputs; ``torch.bmm`` for the fp32 / fp64 GEMMs
of the other input types and for unaligned shapes) with the fused
elementwise / reduction steps of ``csrc/bwd_kernels.cuh`` between them, called
through the C ABI (``avey_bwd_step_v1``):

  PREP      zm (z_tr, padded rows 0), norms      g   = zm zm^T
  SCORES    s = g r_i r_j (.) v (.) mask, den    num = s zm
  EPILOGUE  grad_z_tl, grad_bias, dnum, dden     ds0 = dnum zm^T, dzd = s^T dnum
  DSCORES   dgsym = (dG + dG^T) diag(r), grad_v  dzh = dgsym zm
  FINAL     grad_z_tr

with r = 1 / max(||zm||, norm_eps): every GEMM takes z_tr itself, exact in the
input type, and the norms are applied in fp32 inside the steps. GEMM operands
are bf16 for bf16 inputs (fp32 accumulation and fp32 results) and fp32 / fp64
otherwise: the fp16 range would not hold the products of arbitrary upstream
gradients. fp32 GEMMs follow torch's matmul precision setting (full fp32
unless the caller allows TF32). Under the causal mask s is lower triangular:
g and ds0 are computed only in their 128 x 256 tiles that reach the diagonal
(the steps read nothing above it), and the K loops of num = s zm and
dzd = s^T dnum stop at / start from each row tile's diagonal.
"""

from __future__ import annotations

from typing import List, Optional

import torch

from . import _native
from . import gemm as _gemm

_GEMM_DTYPE = {torch.bfloat16: torch.bfloat16, torch.float16: torch.float32,
               torch.float32: torch.float32, torch.float64: torch.float64}
_DTYPE_IDS = {torch.float32: _native.AVEY_F32, torch.float16: _native.AVEY_F16,
              torch.bfloat16: _native.AVEY_BF16, torch.float64: _native.AVEY_F64}


def _row_strides(t: torch.Tensor):
    return (t.stride(0) if t.shape[0] > 1 else t.shape[1] * t.stride(1)), t.stride(1)


def _unit_last(t: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return t if t is None or t.stride(-1) == 1 else t.contiguous()


def _bmm(a: torch.Tensor, b: torch.Tensor, acc: torch.dtype, mode: int = _gemm.DENSE) -> torch.Tensor:
    """a @ b with results of type `acc`: this library's tcgen05 GEMM for 16-bit
    operands with fp32 results whose bases and strides are 16-byte aligned,
    skipping what the causal `mode` allows; the library GEMM (torch.bmm)
    otherwise (fp32 / fp64 operands, unaligned shapes). Under LOWER_OUT only
    the entries [i][j] with j <= i of the result are defined."""
    if acc == torch.float32 and a.shape[-1] > 0 and b.shape[-1] % 4 == 0 and _gemm.supported(a, b):
        return _gemm.bmm(a, b, mode=mode)
    return torch.bmm(a, b) if a.dtype == acc else torch.bmm(a, b, out_dtype=acc)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def contextualize_backward_impl(z_tr, v, z_tl, bias, valid, grad_out, eps, norm_eps, causal,
                                normalize, activation, needs, packed_out=None):
    """Gradients (z_tr, v, z_tl, bias) of the contextualizer; entries not in
    ``needs`` (or whose input is absent) come back as None. With
    ``packed_out`` (a [B, C, 2d'] tensor), the z_tl and z_tr gradients are
    written into its halves [..., :d'] and [..., d':] instead."""
    if not z_tr.is_cuda:
        raise ValueError('the native backward needs CUDA tensors')
    z_tr, z_tl, grad_out = _unit_last(z_tr), _unit_last(z_tl), _unit_last(grad_out)
    if v is not None and v.stride(1) != 1:
        v = v.contiguous()
    if bias is not None and bias.stride(0) != 1:
        bias = bias.contiguous()
    B, C, d = (int(s) for s in z_tr.shape)
    dev, dt = z_tr.device, z_tr.dtype
    gdt = _GEMM_DTYPE[dt]
    acc = torch.float64 if dt == torch.float64 else torch.float32
    need_z, need_v, need_zl, need_b = (bool(n) for n in needs)
    need_v = need_v and v is not None
    need_zl = need_zl and z_tl is not None
    need_b = need_b and bias is not None

    p = _native.new_bwd_params()
    p.dtype = _DTYPE_IDS[dt]
    p.gemm_dtype = _DTYPE_IDS[gdt]
    p.causal, p.normalize, p.activation = int(bool(causal)), int(bool(normalize)), int(activation)
    p.batch, p.context, p.features = B, C, d
    p.eps, p.norm_eps = float(eps), float(norm_eps)
    p.z_tr = z_tr.data_ptr()
    p.z_tr_batch_stride, p.z_tr_row_stride = _row_strides(z_tr)
    if v is not None:
        p.v = v.data_ptr()
        p.v_row_stride = v.stride(0) if C > 1 else C
    if z_tl is not None:
        p.z_tl = z_tl.data_ptr()
        p.z_tl_batch_stride, p.z_tl_row_stride = _row_strides(z_tl)
    if bias is not None:
        p.bias = bias.data_ptr()
    if valid is not None:
        p.valid = valid.data_ptr()
        p.valid_batch_stride, p.valid_row_stride = valid.stride(0), valid.stride(1)
    p.grad_out = grad_out.data_ptr()
    p.grad_out_batch_stride, p.grad_out_row_stride = _row_strides(grad_out)

    def empty(*shape, dtype):
        return torch.empty(shape, dtype=dtype, device=dev)

    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        norms = empty(B, C, dtype=acc)
        if valid is None and gdt == dt:
            zm = z_tr  # nothing to zero: the GEMMs read z_tr in place (strided)
        else:
            zm = empty(B, C, d, dtype=gdt)
            p.zm = zm.data_ptr()
        p.norms = norms.data_ptr()
        _native.bwd_step(p, _native.BWD_PREP, stream)
        tri = bool(causal)
        g = _bmm(zm, zm.transpose(1, 2), acc, _gemm.LOWER_OUT if tri else _gemm.DENSE)
        s, den = empty(B, C, C, dtype=gdt), empty(B, C, dtype=acc)
        p.g, p.s, p.den = g.data_ptr(), s.data_ptr(), den.data_ptr()
        _native.bwd_step(p, _native.BWD_SCORES, stream)
        num = _bmm(s, zm, acc, _gemm.K_LOWER if tri else _gemm.DENSE)
        dnum, dden = empty(B, C, d, dtype=gdt), empty(B, C, dtype=acc)
        workspace = empty(_native.bwd_workspace_size(p), dtype=torch.uint8)
        if packed_out is not None:
            gz_tl = packed_out[..., :d]
            p.grad_batch_stride, p.grad_row_stride = packed_out.stride(0), packed_out.stride(1)
        else:
            gz_tl = empty(B, C, d, dtype=dt) if need_zl else None
        gbias = empty(d, dtype=dt) if need_b else None
        p.num, p.dnum, p.dden = num.data_ptr(), dnum.data_ptr(), dden.data_ptr()
        p.workspace, p.workspace_bytes = workspace.data_ptr(), workspace.numel()
        p.grad_z_tl, p.grad_bias = _ptr(gz_tl), _ptr(gbias)
        _native.bwd_step(p, _native.BWD_EPILOGUE, stream)
        del num
        gz = gv = None
        if need_z or need_v:
            ds0 = _bmm(dnum, zm.transpose(1, 2), acc, _gemm.LOWER_OUT if tri else _gemm.DENSE)
            dgsym = empty(B, C, C, dtype=gdt)
            gv = empty(C, C, dtype=dt) if need_v else None
            p.ds0, p.dgsym, p.grad_v = ds0.data_ptr(), dgsym.data_ptr(), _ptr(gv)
            _native.bwd_step(p, _native.BWD_DSCORES, stream)
            del ds0, g
            if need_z:
                dzd = _bmm(s.transpose(1, 2), dnum, acc, _gemm.K_UPPER if tri else _gemm.DENSE)
                dzh = _bmm(dgsym, zm, acc)
                gz = packed_out[..., d:] if packed_out is not None else empty(B, C, d, dtype=dt)
                p.dzd, p.dzh, p.grad_z_tr = dzd.data_ptr(), dzh.data_ptr(), gz.data_ptr()
                _native.bwd_step(p, _native.BWD_FINAL, stream)
    return gz, gv, gz_tl, gbias


@torch.library.custom_op('avey_b200::contextualize_backward', mutates_args=())
def contextualize_backward(z_tr: torch.Tensor, v: Optional[torch.Tensor],
                           z_tl: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                           valid: Optional[torch.Tensor], grad_out: torch.Tensor, eps: float,
                           norm_eps: float, causal: bool, normalize: bool, activation: int,
                           needs: List[bool]) -> List[torch.Tensor]:
    """Native backward as one op: [grad_z_tr, grad_v, grad_z_tl, grad_bias],
    an empty tensor standing for a gradient that was not requested."""
    grads = contextualize_backward_impl(z_tr, v, z_tl, bias, valid, grad_out, eps, norm_eps,
                                        causal, normalize, activation, needs)
    return [t if t is not None else z_tr.new_empty(0) for t in grads]


@contextualize_backward.register_fake
def _contextualize_backward_fake(z_tr, v, z_tl, bias, valid, grad_out, eps, norm_eps, causal,
                                 normalize, activation, needs):
    shapes = (z_tr.shape, None if v is None else v.shape,
              None if z_tl is None else z_tl.shape, None if bias is None else bias.shape)
    return [z_tr.new_empty(s) if (s is not None and n) else z_tr.new_empty(0)
            for s, n in zip(shapes, needs)]


def _setup_context(ctx, inputs, output):
    z_tr, v, z_tl, bias, valid, eps, norm_eps, causal, normalize, activation, _variant = inputs
    ctx.save_for_backward(z_tr, v, z_tl, bias, valid)
    ctx.cfg = (eps, norm_eps, causal, normalize, activation)


def _backward(ctx, grad):
    z_tr, v, z_tl, bias, valid = ctx.saved_tensors
    needs = [bool(n) for n in ctx.needs_input_grad[:4]]
    grads = contextualize_backward(z_tr, v, z_tl, bias, valid, grad, *ctx.cfg, needs)
    out = [t if (n and t.numel()) else None for t, n in zip(grads, needs)]
    return (*out, None, None, None, None, None, None, None)


def register() -> None:
    """Attach the native backward to ``avey_b200::contextualize`` (once)."""
    torch.library.register_autograd('avey_b200::contextualize', _backward,
                                    setup_context=_setup_context)


# ---------------------------------------------------------------------------
# Packed form: z_tl and z_tr are the halves [..., :d'] and [..., d':] of one
# [B, C, 2d'] tensor x (the enricher output split into head and tail). Taking
# x as the op's input gives autograd one gradient for x, written in place by
# the backward steps, instead of two half-size gradients that autograd would
# scatter into zero-filled copies of x and add.

@torch.library.custom_op('avey_b200::contextualize_packed_backward', mutates_args=())
def contextualize_packed_backward(x: torch.Tensor, v: Optional[torch.Tensor],
                                  bias: Optional[torch.Tensor], valid: Optional[torch.Tensor],
                                  grad_out: torch.Tensor, eps: float, norm_eps: float,
                                  causal: bool, normalize: bool, activation: int,
                                  needs: List[bool]) -> List[torch.Tensor]:
    """[grad_x, grad_v, grad_bias] of ``avey_b200::contextualize_packed``."""
    d = x.shape[-1] // 2
    gx = torch.empty_like(x, memory_format=torch.contiguous_format) if needs[0] else None
    _, gv, _, gb = contextualize_backward_impl(
        x[..., d:], v, x[..., :d], bias, valid, grad_out, eps, norm_eps, causal, normalize,
        activation, [needs[0], needs[1], needs[0], needs[2]], packed_out=gx)
    return [t if t is not None else x.new_empty(0) for t in (gx, gv, gb)]


@contextualize_packed_backward.register_fake
def _contextualize_packed_backward_fake(x, v, bias, valid, grad_out, eps, norm_eps, causal,
                                        normalize, activation, needs):
    shapes = (x.shape, None if v is None else v.shape, None if bias is None else bias.shape)
    return [x.new_empty(s) if (s is not None and n) else x.new_empty(0)
            for s, n in zip(shapes, needs)]


def _setup_context_packed(ctx, inputs, output):
    x, v, bias, valid, eps, norm_eps, causal, normalize, activation = inputs
    ctx.save_for_backward(x, v, bias, valid)
    ctx.cfg = (eps, norm_eps, causal, normalize, activation)


def _backward_packed(ctx, grad):
    x, v, bias, valid = ctx.saved_tensors
    needs = [bool(n) for n in ctx.needs_input_grad[:3]]
    grads = contextualize_packed_backward(x, v, bias, valid, grad, *ctx.cfg, needs)
    out = [t if (n and t.numel()) else None for t, n in zip(grads, needs)]
    return (*out, None, None, None, None, None, None, None)


def register_packed() -> None:
    """Attach the native backward to ``avey_b200::contextualize_packed``."""
    torch.library.register_autograd('avey_b200::contextualize_packed', _backward_packed,
                                    setup_context=_setup_context_packed)
