"""The batched tcgen05 matrix product (``avey_gemm_v1`` through
``avey_kernel_b200.gemm``) on a B200.

Reference: the fp64 product of the same 16-bit operands (bf16 / f16 products
are exact in fp32, so the kernel's only error is its fp32 summation order):
|c - ref| <= 1e-5 * (|a| @ |b|) + 1e-6 elementwise. Covered: both majors of
each operand (transposed views, no copies), partial tiles on every edge, K
not a multiple of the 64-wide K block, shared (batch stride 0) operands, the
causal modes (LOWER_OUT checked on j <= i; the K-range modes on triangular A,
bit for bit against DENSE), and the 16-bit epilogue (bias, activation, gate,
row sums of squares of the stored values).
"""

import zlib

import pytest
import torch

from avey_kernel_b200 import _native, gemm

pytestmark = pytest.mark.gpu
DEV = 'cuda'


@pytest.fixture(autouse=True)
def _device_status_clean():
    _native.device_status(clear=True)
    yield
    assert _native.device_status(clear=True) == 0


def operand(shape, dtype, major, gen, kind):
    """A [B, r, c] operand whose major layout is `major` ('row': last dim
    contiguous; 'col': the view of a transposed contiguous tensor)."""
    b, r, c = shape
    if major == 'row':
        return torch.randn(b, r, c, generator=gen).to(dtype).to(DEV)
    return torch.randn(b, c, r, generator=gen).to(dtype).to(DEV).transpose(1, 2)


def check(c, a, b, lower_only=False):
    ref = torch.bmm(a.double(), b.double())
    bound = 1e-5 * torch.bmm(a.double().abs(), b.double().abs()) + 1e-6
    err = (c.double() - ref).abs() - bound
    if lower_only:
        m, n = c.shape[1], c.shape[2]
        keep = torch.arange(n, device=DEV)[None, :] <= torch.arange(m, device=DEV)[:, None]
        err = err[:, keep]
    assert float(err.max()) <= 0.0, float(err.max())


KERNELS = [gemm.KERNEL_SINGLE, gemm.KERNEL_PAIR]


@pytest.mark.parametrize('kernel', KERNELS)
@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('a_major', ['row', 'col'])
@pytest.mark.parametrize('b_major', ['row', 'col'])
@pytest.mark.parametrize('shape', [(3, 200, 296, 72), (2, 512, 768, 512), (1, 128, 256, 64),
                                   (2, 40, 24, 136), (2, 384, 640, 192)])
def test_dense_matches_fp64(kernel, dtype, a_major, b_major, shape):
    g = torch.Generator().manual_seed(zlib.crc32(repr((a_major, b_major, shape)).encode()))
    bt, m, n, k = shape
    a = operand((bt, m, k), dtype, a_major, g, 'a')
    b = operand((bt, k, n), dtype, b_major, g, 'b')
    assert gemm.supported(a, b)
    before = _native.launch_count()
    c = gemm.bmm(a, b, kernel=kernel)
    torch.cuda.synchronize()
    assert _native.launch_count() == before + 1
    check(c, a, b)


@pytest.mark.parametrize('shape', [(64, 512, 768, 512), (4, 1000, 1536, 768)])
def test_pair_and_single_kernels_agree(shape):
    """The CTA-pair kernel (256 x 256 tiles) and the single-CTA kernel give the
    same products up to fp32 summation order, on backward- and enricher-sized
    shapes (many tiles per CTA: the accumulator double buffering wraps)."""
    g = torch.Generator().manual_seed(shape[1])
    bt, m, n, k = shape
    a = torch.randn(bt, m, k, generator=g).to(torch.bfloat16).to(DEV)
    b = torch.randn(bt, n, k, generator=g).to(torch.bfloat16).to(DEV).transpose(1, 2)
    c1 = gemm.bmm(a, b, kernel=gemm.KERNEL_SINGLE)
    c2 = gemm.bmm(a, b, kernel=gemm.KERNEL_PAIR)
    check(c2, a, b)
    torch.testing.assert_close(c1, c2, rtol=1e-5, atol=1e-4)


def test_shared_operand_across_batch():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 300, 128, generator=g).to(torch.bfloat16).to(DEV)
    w = torch.randn(1, 128, 384, generator=g).to(torch.bfloat16).to(DEV).expand(4, 128, 384)
    assert w.stride(0) == 0
    check(gemm.bmm(x, w), x, w)


@pytest.mark.parametrize('kernel', KERNELS)
@pytest.mark.parametrize('ctx,feat', [(512, 768), (384, 256), (200, 136)])
def test_causal_modes(kernel, ctx, feat):
    """The backward's five products under the causal mask: g / ds0 keep only
    j <= i, num = s z and dzd = s^T dnum skip the zero half of s exactly."""
    g = torch.Generator().manual_seed(ctx)
    bt = 3
    z = torch.randn(bt, ctx, feat, generator=g).to(torch.bfloat16).to(DEV)
    dn = torch.randn(bt, ctx, feat, generator=g).to(torch.bfloat16).to(DEV)
    s = torch.randn(bt, ctx, ctx, generator=g).to(torch.bfloat16).to(DEV).tril()
    # Garbage in the skipped tiles must stay there: prefill the output with NaN.
    out = torch.full((bt, ctx, ctx), float('nan'), device=DEV)
    gm = gemm.bmm(z, z.transpose(1, 2), mode=gemm.LOWER_OUT, out=out, kernel=kernel)
    check(gm, z, z.transpose(1, 2), lower_only=True)
    num = gemm.bmm(s, z, mode=gemm.K_LOWER, kernel=kernel)
    assert torch.equal(num, gemm.bmm(s, z, kernel=kernel))
    check(num, s, z)
    dzd = gemm.bmm(s.transpose(1, 2), dn, mode=gemm.K_UPPER, kernel=kernel)
    assert torch.equal(dzd, gemm.bmm(s.transpose(1, 2), dn, kernel=kernel))
    check(dzd, s.transpose(1, 2), dn)


ACTS = {0: lambda x: x, 1: torch.relu, 2: lambda x: torch.relu(x) ** 2, 3: torch.nn.functional.silu,
        4: lambda x: torch.nn.functional.gelu(x, approximate='tanh')}


@pytest.mark.parametrize('kernel', KERNELS)
@pytest.mark.parametrize('act', [0, 1, 2, 3, 4])
@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
def test_16bit_epilogue(kernel, act, dtype):
    """out = act(x w^T + bias) (.) gate in the operand type, and the row sums of
    squares of the stored outputs of columns >= col0 in 128-column planes."""
    import ctypes

    gen = torch.Generator().manual_seed(act)
    bt, m, n, k, col0 = 2, 300, 640, 192, 256
    x = torch.randn(bt, m, k, generator=gen).to(dtype).to(DEV)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).to(dtype).to(DEV)
    bias = (torch.randn(n, generator=gen) * 0.1).to(dtype).to(DEV)
    gate = torch.randn(bt, m, n, generator=gen).to(dtype).to(DEV)
    out = torch.empty(bt, m, n, dtype=dtype, device=DEV)
    planes = (n - col0 + 127) // 128
    ss = torch.full((planes, bt * m), float('nan'), device=DEV)
    wt = w.t().unsqueeze(0).expand(bt, k, n)
    p = gemm._params(x, wt, out, gemm.DENSE, kernel)
    p.bias, p.gate = bias.data_ptr(), gate.data_ptr()
    p.gate_batch_stride, p.gate_ld = gate.stride(0), gate.stride(1)
    p.activation, p.sumsq_col0, p.sumsq = act, col0, ss.data_ptr()
    _native.gemm(p, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = ACTS[act](torch.bmm(x.double(), wt.double()) + bias.double()) * gate.double()
    scale = float(ref.abs().max())
    assert float((out.double() - ref).abs().max()) <= 1e-2 * scale
    stored = out.float()[..., col0:] ** 2
    for pi in range(planes):
        want = stored[..., 128 * pi:128 * pi + 128].sum(-1).reshape(-1)
        torch.testing.assert_close(ss[pi], want, rtol=1e-5, atol=1e-6)
    assert ctypes.sizeof(_native.AveyGemmParams) > 0


def test_rejects_unaligned_operands():
    x = torch.randn(2, 64, 36, device=DEV).to(torch.bfloat16)  # rows of 72 bytes
    assert not gemm.supported(x, x.transpose(1, 2))
    with pytest.raises(ValueError):
        gemm.bmm(x, x.transpose(1, 2))
