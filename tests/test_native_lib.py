"""The C-ABI library: it loads, exports what the header declares, and its
host-side logic (validation, kernel plan) behaves -- no GPU needed."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

from avey_kernel_b200 import _native, ops

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'avey_b200.h'


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r'AVEY_API\s+[\w\s\*]+?\b(avey_\w+)\s*\(', text)))


def test_library_loads_and_reports_abi_version():
    dll = _native.lib()
    assert dll.avey_abi_version() == _native.ABI_VERSION == 5


def test_every_header_function_is_exported():
    declared = header_functions()
    assert declared == sorted(_native.EXPORTS)
    dll = _native.lib()
    for name in declared:
        assert hasattr(dll, name), name
    nm = subprocess.run(['nm', '-D', '--defined-only', str(_native.library_path())],
                        capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r' T (avey_\w+)', nm))
    assert set(declared) <= exported


def _params(shape=(2, 64, 128), dtype=torch.bfloat16, **kw):
    z = torch.randn(*shape).to(dtype)
    out = torch.empty_like(z)
    return ops.build_params(z, kw.pop('v', None), kw.pop('z_tl', None), None, None, out,
                            eps=kw.pop('eps', 1e-6), norm_eps=1e-12, causal=True,
                            normalize=False, activation_id=0, kernel=kw.pop('kernel', 0)), (z, out)


def test_struct_size_guard():
    p, _keep = _params()
    p.struct_size = 8
    with pytest.raises(_native.NativeError, match='struct_size'):
        _native.plan(p)


@pytest.mark.parametrize('field,value,match', [
    ('batch', 0, 'must be >= 1'),
    ('features', 0, 'must be >= 1'),
    ('activation', 7, 'activation'),
    ('kernel', 9, 'kernel'),
    ('eps', 0.0, 'finite and positive'),
    ('norm_eps', float('nan'), 'finite and positive'),
    ('dtype', 11, 'dtype'),
    ('z_tr_row_stride', 3, 'row strides'),
])
def test_invalid_arguments_are_rejected_before_any_launch(field, value, match):
    p, _keep = _params()
    setattr(p, field, value)
    before = _native.launch_count()
    with pytest.raises(_native.NativeError, match=match) as info:
        _native.forward(p, 0)
    assert info.value.status == -1
    assert _native.launch_count() == before


def test_null_required_pointer():
    p, _keep = _params()
    p.z_tr = None
    with pytest.raises(_native.NativeError, match='required'):
        _native.plan(p)


def test_plan_chooses_tcgen05_for_aligned_16bit_inputs():
    z = torch.randn(4, 512, 768).to(torch.bfloat16)
    plan = ops.plan(z, torch.randn(512, 512).to(torch.bfloat16), z_tl=z)
    assert plan.kernel == _native.KERNEL_TCGEN05 and plan.reason == 0
    assert plan.grid == 4 * 4 and plan.block == 384 and plan.launches == 1
    assert 200_000 < plan.smem_bytes <= 232_448


def test_plan_accepts_head_tail_views_without_copy():
    x = torch.randn(2, 256, 2 * 384).to(torch.bfloat16)
    head, tail = x[..., :384], x[..., 384:]
    plan = ops.plan(tail, z_tl=head, causal=False, normalize=True)
    assert plan.kernel == _native.KERNEL_TCGEN05


@pytest.mark.parametrize('shape,dtype,reason', [
    ((2, 35, 133), torch.float32, 3),    # 133 fp32 features: rows not 16-byte aligned
    ((2, 35, 37), torch.bfloat16, 3),    # 37 features: rows not 16-byte aligned
    ((1, 8200, 64), torch.bfloat16, 2),  # more than 8192 tokens
    ((1, 8200, 64), torch.float32, 2),
    ((2, 35, 40), torch.float64, 1),     # fp64 -> CUDA-core kernel
])
def test_plan_falls_back_to_cuda_core_kernel(shape, dtype, reason):
    z = torch.randn(*shape).to(dtype)
    plan = ops.plan(z)
    assert plan.kernel == _native.KERNEL_SIMT and plan.reason == reason


@pytest.mark.parametrize('shape,items', [((16, 256, 128), 2), ((64, 512, 768), 6), ((1, 1100, 72), 25)])
def test_plan_runs_fp32_on_the_3xtf32_kernel_pair(shape, items):
    # fp32: tf_gram_p per (query tile, key group of 256) and tf_pv, no pre-pass
    # (the split of each staged tile sums the squares); the workspace holds P
    # as fp32.
    z = torch.randn(*shape)
    b, n, d = shape
    plan = ops.plan(z, torch.randn(n, n), z_tl=z)
    assert plan.kernel == _native.KERNEL_TCGEN05 and plan.reason == 0
    assert plan.launches == 2 and plan.block == 256 and plan.grid == b * items
    assert 190_000 < plan.smem_bytes <= 232_448
    params = ops.build_params(z, torch.randn(n, n), z, None, None, torch.empty_like(z), eps=1e-6,
                              norm_eps=1e-12, causal=True, normalize=False, activation_id=0)
    cp = -(-n // 64) * 64
    assert _native.workspace_size(params) >= b * n * cp * 4


@pytest.mark.parametrize('shape,dtype,small', [
    ((2, 256, 128), torch.float32, True),     # config 1: 64 CTA pairs of 8 query rows
    ((4, 512, 128), torch.float32, True),     # 256 query tiles: within 4 waves of 74
    ((5, 512, 128), torch.float32, False),    # 320 query tiles: 3xTF32 pair
    ((18, 64, 128), torch.float32, True),     # 144 tiles of short rows: within 2 waves
    ((19, 64, 128), torch.float32, False),    # 152 tiles of short rows: 3xTF32 pair
    ((2, 96, 256), torch.float32, True),      # rows of 1 KB (64-key blocks)
    ((8, 512, 256), torch.float32, False),    # 512 query tiles: 3xTF32 pair
    ((2, 256, 72), torch.float32, False),     # features not a multiple of 32
    ((2, 256, 512), torch.float32, False),    # rows above 1 KB
    ((2, 600, 64), torch.float32, False),     # above 512 tokens
    ((2, 256, 128), torch.bfloat16, False),   # 16-bit inputs keep the fused tcgen05 kernel
])
def test_plan_runs_small_fp32_problems_on_the_8_row_kernel(shape, dtype, small):
    z = torch.randn(*shape).to(dtype)
    b, n, _ = shape
    v = torch.randn(n, n).to(dtype)
    plan = ops.plan(z, v, z_tl=z)
    if small:
        assert plan.kernel == _native.KERNEL_SIMT and plan.reason == _native.REASON_SMALL
        assert plan.launches == 1 and plan.block == 512 and plan.grid == 2 * b * -(-n // 8)
        assert plan.smem_bytes <= 232_448
        # Asked for, the 3xTF32 pair still takes these inputs.
        forced = ops.plan(z, v, z_tl=z, kernel=_native.KERNEL_TCGEN05)
        assert forced.kernel == _native.KERNEL_TCGEN05 and forced.launches == 2
    else:
        assert plan.kernel == _native.KERNEL_TCGEN05 and plan.reason == 0


def test_plan_takes_the_long_context_tcgen05_path_above_512_tokens():
    z = torch.randn(2, 2048, 1024).to(torch.bfloat16)
    plan = ops.plan(z, torch.randn(2048, 2048).to(torch.bfloat16), z_tl=z)
    assert plan.kernel == _native.KERNEL_TCGEN05 and plan.reason == 0
    # pre-pass, G/P per (query tile, key group), O = P Z: 72 items per batch row
    # (query tile t has ceil((t + 1) / 2) groups of 256 keys)
    assert plan.launches == 3 and plan.grid == 2 * 72 and plan.block == 256
    assert plan.smem_bytes <= 232_448


def test_long_context_workspace_holds_sums_partial_sums_and_p():
    b, n, d = 3, 700, 128
    z = torch.randn(b, n, d).to(torch.bfloat16)
    out = torch.empty_like(z)
    p = ops.build_params(z, None, None, None, None, out, eps=1e-6, norm_eps=1e-12, causal=False,
                         normalize=True, activation_id=0)
    al = lambda x: (x + 255) // 256 * 256
    groups, padded = (n + 255) // 256, (n + 63) // 64 * 64
    assert _native.workspace_size(p) == al(b * n * 4) + al(b * groups * n * 4) + b * n * padded * 2


def test_forcing_tcgen05_on_unsupported_inputs_fails():
    z = torch.randn(2, 35, 37)
    with pytest.raises(_native.NativeError) as info:
        ops.plan(z, kernel=_native.KERNEL_TCGEN05)
    assert info.value.status == -3


def test_ctypes_struct_matches_header_field_order():
    text = HEADER.read_text()
    body = text[text.index('typedef struct AveyFwdParams'):text.index('} AveyFwdParams;')]
    names = re.findall(r'\b(\w+)\s*[;,]', re.sub(r'/\*.*?\*/', '', body, flags=re.S))
    names = [n for n in names if n not in ('AveyFwdParams',)]
    assert names == [f for f, _ in _native.AveyFwdParams._fields_]
    # The library rejects any other size (test_struct_size_guard); 200 bytes on LP64.
    assert ctypes.sizeof(_native.AveyFwdParams) == 208


def test_workspace_size_by_path():
    # The fused tcgen05 kernel (16-bit, up to 512 tokens) sums the rows'
    # squares itself: no workspace.
    z = torch.randn(3, 384, 256).to(torch.bfloat16)
    out = torch.empty_like(z)
    p = ops.build_params(z, None, None, None, None, out, eps=1e-6, norm_eps=1e-12, causal=False,
                         normalize=True, activation_id=0)
    assert ops.plan(z, causal=False, normalize=True).kernel == _native.KERNEL_TCGEN05
    assert _native.workspace_size(p) == 0
    # Above 512 tokens: row sums, partial row sums and P (bf16, rows padded to 64 keys).
    zl = torch.randn(2, 600, 64).to(torch.bfloat16)
    p = ops.build_params(zl, None, None, None, None, zl.clone(), eps=1e-6, norm_eps=1e-12,
                         causal=False, normalize=True, activation_id=0)
    assert _native.workspace_size(p) >= 2 * 600 * 640 * 2 + 2 * 600 * 4
    # fp32 runs the 3xTF32 kernel pair: partial row sums and P (fp32, rows
    # padded to 64 keys) follow the per-row floats.
    z32 = torch.randn(8, 384, 256)
    p = ops.build_params(z32, None, None, None, None, z32.clone(), eps=1e-6, norm_eps=1e-12,
                         causal=False, normalize=True, activation_id=0)
    assert _native.workspace_size(p) >= 8 * 384 * 384 * 4 + 8 * 384 * 4
    # Small fp32 problems run the 8-row CUDA-core kernel, which needs none.
    p = ops.build_params(z.float(), None, None, None, None, z.float(), eps=1e-6, norm_eps=1e-12,
                         causal=False, normalize=True, activation_id=0)
    assert _native.workspace_size(p) == 0
    # Inputs the CUDA-core kernels take need none.
    z37 = torch.randn(3, 384, 37)
    p = ops.build_params(z37, None, None, None, None, z37.clone(), eps=1e-6, norm_eps=1e-12,
                         causal=False, normalize=True, activation_id=0)
    assert _native.workspace_size(p) == 0


def _bwd_params(b=2, c=64, d=128, dtype=_native.AVEY_BF16, gemm=_native.AVEY_BF16, with_v=True):
    p = _native.new_bwd_params()
    p.dtype, p.gemm_dtype = dtype, gemm
    p.batch, p.context, p.features = b, c, d
    p.eps, p.norm_eps = 1e-6, 1e-12
    p.causal = 1
    p.z_tr = 0x1000  # host-side checks only: nothing is dereferenced or launched
    p.z_tr_batch_stride, p.z_tr_row_stride = c * d, d
    if with_v:
        p.v, p.v_row_stride = 0x2000, c
    return p


def test_backward_workspace_size_covers_dbias_and_dv_partial_sums():
    # Vector form (rows of multiples of 8, aligned): 32 rows per epilogue block,
    # one fp32 partial row of d' per block; dV: one [C, C] partial per batch group.
    p = _bwd_params(b=2, c=64, d=128)
    epi = (2 * 64 // 32) * 128
    pairs = 2 * 3 // 2  # 64 tokens = 2 tiles of 32: (0,0), (0,1), (1,1)
    groups = min(2, -(-1184 // pairs), 16)
    assert _native.bwd_workspace_size(p) == max(epi, groups * 64 * 64) * 4
    p64 = _bwd_params(dtype=_native.AVEY_F64, gemm=_native.AVEY_F64, with_v=False)
    assert _native.bwd_workspace_size(p64) == (2 * 64 // 64) * 128 * 8  # scalar form, fp64


@pytest.mark.parametrize('field,value,match', [
    ('gemm_dtype', _native.AVEY_F32, 'gemm_dtype'),
    ('batch', 0, 'out of range'),
    ('activation', 5, 'activation'),
    ('eps', -1.0, 'finite and positive'),
    ('z_tr_row_stride', 4, 'strides'),
    ('grad_row_stride', 8, 'strides'),
    ('struct_size', 12, 'struct_size'),
])
def test_backward_rejects_invalid_arguments_before_any_launch(field, value, match):
    p = _bwd_params()
    setattr(p, field, value)
    before = _native.launch_count()
    with pytest.raises(_native.NativeError, match=match):
        _native.bwd_step(p, _native.BWD_PREP, 0)
    assert _native.launch_count() == before


def test_backward_steps_check_their_buffers_and_step_ids():
    p = _bwd_params()
    for step, match in ((_native.BWD_PREP, 'prep needs'), (_native.BWD_SCORES, 'scores needs'),
                        (_native.BWD_EPILOGUE, 'epilogue needs'), (_native.BWD_DSCORES, 'dscores needs'),
                        (_native.BWD_FINAL, 'final needs'), (9, 'unknown backward step')):
        with pytest.raises(_native.NativeError, match=match):
            _native.bwd_step(p, step, 0)


@pytest.mark.parametrize('step', [_native.BWD_PREP, _native.BWD_FINAL])
def test_backward_omits_zm_only_without_padding_and_with_the_input_gemm_type(step):
    # zm may be NULL (the steps then read z_tr) only when it would equal z_tr.
    for dtype, gemm, padded in ((_native.AVEY_BF16, _native.AVEY_BF16, True),
                                (_native.AVEY_F16, _native.AVEY_F32, False)):
        p = _bwd_params(dtype=dtype, gemm=gemm)
        p.norms, p.dzh, p.dzd, p.grad_z_tr = 0x3000, 0x4000, 0x5000, 0x6000
        if padded:
            p.valid, p.valid_batch_stride, p.valid_row_stride = 0x7000, 64, 1
        before = _native.launch_count()
        with pytest.raises(_native.NativeError, match='zm may be NULL only'):
            _native.bwd_step(p, step, 0)
        assert _native.launch_count() == before


def test_mask_as_valid_and_lengths_together_is_rejected():
    p, _keep = _params()
    valid = torch.ones(2, 64, dtype=torch.bool)
    lengths = torch.full((2,), 64, dtype=torch.int32)
    p.valid, p.lengths = valid.data_ptr(), lengths.data_ptr()
    with pytest.raises(_native.NativeError, match='not both'):
        _native.plan(p)


def _gemm_params(**kw):
    """A valid AveyGemmParams for [2, 64, 32] x [2, 32, 48] bf16 (host pointers
    are never dereferenced: validation fails or passes before any launch)."""
    p = _native.AveyGemmParams()
    p.struct_size = ctypes.sizeof(_native.AveyGemmParams)
    p.dtype, p.out_dtype, p.mode = _native.AVEY_BF16, _native.AVEY_F32, 0
    p.batch, p.m, p.n, p.k = 2, 64, 48, 32
    p.a, p.a_batch_stride, p.a_ld, p.a_major = 1 << 20, 64 * 32, 32, 0
    p.b, p.b_batch_stride, p.b_ld, p.b_major = 2 << 20, 48 * 32, 32, 0
    p.c, p.c_batch_stride, p.c_ld = 3 << 20, 64 * 48, 48
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize('field,value,match', [
    ('struct_size', 8, 'struct_size'),
    ('dtype', _native.AVEY_F32, 'bf16 or f16'),
    ('out_dtype', _native.AVEY_F16, 'out_dtype'),
    ('mode', 9, 'mode'),
    ('k', 0, r'\[1, 2\^24\]'),
    ('a_major', 3, 'a_major'),
    ('a_ld', 16, 'leading dimensions'),
    ('b_ld', 36, 'whole 16-byte units'),
    ('a', (1 << 20) + 8, 'aligned'),
    ('activation', 2, 'need a 16-bit output'),
    ('kernel', 5, 'GEMM kernel'),
])
def test_gemm_arguments_are_rejected_before_any_launch(field, value, match):
    p = _gemm_params(**{field: value})
    before = _native.launch_count()
    with pytest.raises(_native.NativeError, match=match) as info:
        _native.gemm(p, 0)
    assert info.value.status == -1
    assert _native.launch_count() == before


def test_gemm_sums_need_a_128_column_boundary():
    p = _gemm_params(out_dtype=_native.AVEY_BF16, n=512, c_ld=512, sumsq=4 << 20, sumsq_col0=100)
    with pytest.raises(_native.NativeError, match='multiple of 128'):
        _native.gemm(p, 0)


def test_presummed_forward_checks_its_planes():
    p, _keep = _params()
    with pytest.raises(_native.NativeError, match='planes'):
        _native.forward_presummed(p, 1 << 20, 0, 0)
    with pytest.raises(_native.NativeError, match='planes'):
        _native.forward_presummed(p, 0, 2, 0)
