"""The drop-in API: signatures, validation errors, the differentiable PyTorch
path, and custom-op tracing without a GPU (mirrors the reference's
tests/test_contextualizer.py, tests/test_symbolic_tile.py and
tests/test_autotune.py:25-45)."""

import io
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import oracle
from avey_kernel_b200 import avey, avey_b, ops
from fixtures import load_cases, oracle_kwargs, to_torch
from helpers import TOL, norm_rel_err, to_numpy

CASES = load_cases()
ROOT = Path(__file__).resolve().parents[1]
FP32_TOL = dict(rtol=1.3e-6, atol=1e-5)


def test_package_exports():
    import avey_kernel_b200
    assert avey_kernel_b200.__all__ == ['avey', 'avey_b']


def test_weight_orientation_and_causality():
    z = torch.tensor([[[1., 0.], [0., 2.], [3., 0.]]])
    v = torch.tensor([[2., 7., 11.], [13., 3., 17.], [5., 19., 4.]])
    torch.testing.assert_close(avey(z, v, backend='torch'),
                               torch.tensor([[[2., 0.], [0., 6.], [17., 0.]]]))
    torch.testing.assert_close(avey(z, v, causal=False, backend='torch')[0, 0],
                               torch.tensor([35., 0.]))


def test_avey_b_divides_before_bias_activation_and_gate():
    z = torch.tensor([[[1., 0.], [3., 0.]]])
    gate = torch.tensor([[[2., 3.], [4., 5.]]])
    out = avey_b(z, z_tl=gate, bias=torch.tensor([-3., 1.]), activation='relu', eps=2.,
                 backend='torch')
    torch.testing.assert_close(out, torch.tensor([[[0., 3.], [0., 5.]]]))


def test_zero_rows_and_padding_do_not_leak_bias():
    z = torch.tensor([[[0., 0.], [2., 0.], [100., 100.]]])
    out = avey_b(z, valid=torch.tensor([[True, True, False]]), bias=torch.ones(2),
                 backend='torch')
    torch.testing.assert_close(out, torch.tensor([[[1., 1.], [3., 1.], [0., 0.]]]))


def test_signed_denominator():
    z = torch.tensor([[[1., 0.], [-2., 0.]]], dtype=torch.float64)
    torch.testing.assert_close(avey_b(z, eps=0.5, backend='torch'),
                               torch.tensor([[[6., 0.], [-6., 0.]]], dtype=torch.float64))


def test_gradcheck_on_the_torch_path():
    z = torch.rand(1, 3, 2, dtype=torch.float64, requires_grad=True)
    v = torch.rand(3, 3, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda x, w: avey(x, w, backend='torch'), (z, v))
    assert torch.autograd.gradcheck(lambda x: avey_b(x, backend='torch'), (z,))


def test_nan_padding_cannot_contaminate_gradients():
    for normalized in (False, True):
        z = torch.tensor([[[1., 2.], [3., 4.], [float('nan'), float('nan')]]], requires_grad=True)
        gate = torch.tensor([[[1., 1.], [1., 1.], [float('nan'), float('nan')]]],
                            requires_grad=True)
        valid = torch.tensor([[True, True, False]])
        out = (avey_b(z, z_tl=gate, valid=valid, backend='torch') if normalized
               else avey(z, torch.ones(3, 3), z_tl=gate, valid=valid, backend='torch'))
        out.sum().backward()
        assert torch.isfinite(z.grad).all() and torch.isfinite(gate.grad).all()
        torch.testing.assert_close(z.grad[:, -1], torch.zeros(1, 2))
        torch.testing.assert_close(gate.grad[:, -1], torch.zeros(1, 2))


def test_input_contract():
    z = torch.ones(1, 3, 2)
    bad_calls = [
        lambda: avey(z, torch.ones(2, 2)),
        lambda: avey(z, None),
        lambda: avey_b(z, eps=0.),
        lambda: avey_b(z, norm_eps=float('inf')),
        lambda: avey_b(z, activation='softmax'),
        lambda: avey_b(z, backend='unknown'),
        lambda: avey_b(z, valid=torch.ones(1, 3)),
        lambda: avey_b(torch.ones(0, 3, 2)),
        lambda: avey_b(torch.ones(3, 2)),
        lambda: avey_b(z.int()),
        lambda: avey_b(z, bias=torch.ones(3)),
        lambda: avey_b(z, z_tl=torch.ones(1, 3, 2, dtype=torch.float64)),
        lambda: avey_b(z, autotune=1),
    ]
    for call in bad_calls:
        with pytest.raises(ValueError):
            call()
    for output_tile in (16, 256, 32.0):
        with pytest.raises(ValueError):
            avey_b(z, output_tile=output_tile)


def test_auto_backend_preserves_autograd_on_cpu():
    z = torch.ones(1, 3, 2, requires_grad=True)
    avey_b(z).sum().backward()
    assert z.grad is not None
    x = torch.rand(1, 5, 7, requires_grad=True)
    out = avey_b(x, autotune=True)
    torch.testing.assert_close(out, avey_b(x, backend='torch'))


def test_native_backend_rejects_cpu_inputs():
    with pytest.raises(ValueError, match='CUDA tensors'):
        avey_b(torch.rand(1, 5, 8), backend='cuda')
    with pytest.raises(ValueError, match='CUDA tensors'):
        avey_b(torch.rand(1, 5, 8, requires_grad=True), backend='cuda')


def test_triton_backend_keeps_the_reference_rules_on_cpu():
    # The reference's backend='triton' wants CUDA fp16/bf16/fp32 inference
    # inputs (ops.py:96-103) and raises ValueError otherwise.
    with pytest.raises(ValueError, match='inference inputs'):
        avey_b(torch.rand(1, 5, 8), backend='triton')
    with pytest.raises(ValueError, match='inference inputs'):
        avey_b(torch.rand(1, 5, 8, requires_grad=True), backend='triton')


REFERENCE_TESTS = Path('/root/reference/tests/test_contextualizer.py')


@pytest.mark.skipif(not REFERENCE_TESTS.exists(), reason='the reference checkout is not mounted')
def test_the_reference_contract_tests_pass_against_this_package():
    # Runs the reference's own public-API tests (tests/test_contextualizer.py:
    # orientation, ordering, padding, signed sums, gradients, NaN padding, the
    # input contract, autograd under 'auto') with `avey_kernels` bound to this
    # package, on CPU tensors.
    import importlib.util
    import types
    import unittest

    import avey_kernel_b200
    shim = types.ModuleType('avey_kernels')
    shim.avey, shim.avey_b = avey_kernel_b200.avey, avey_kernel_b200.avey_b
    saved = sys.modules.get('avey_kernels')
    sys.modules['avey_kernels'] = shim
    try:
        spec = importlib.util.spec_from_file_location('reference_test_contextualizer',
                                                      REFERENCE_TESTS)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        suite = unittest.defaultTestLoader.loadTestsFromModule(mod)
        result = unittest.TextTestRunner(stream=io.StringIO(), verbosity=0).run(suite)
    finally:
        if saved is None:
            sys.modules.pop('avey_kernels', None)
        else:
            sys.modules['avey_kernels'] = saved
    assert result.testsRun >= 8
    assert result.wasSuccessful(), [str(f[1])[-400:] for f in result.failures + result.errors]


@pytest.mark.parametrize('case', CASES, ids=[c['name'] for c in CASES])
def test_torch_path_matches_oracle(case):
    t = to_torch(case)
    kw = oracle_kwargs(case)
    if case['op'] == 'avey':
        out = avey(t['z_tr'], t['v'], z_tl=t['z_tl'], bias=t['bias'], valid=t['valid'],
                   causal=kw['causal'], activation=kw['activation'], backend='torch')
    else:
        out = avey_b(t['z_tr'], z_tl=t['z_tl'], bias=t['bias'], valid=t['valid'], eps=kw['eps'],
                     activation=kw['activation'], backend='torch')
    assert out.dtype == t['z_tr'].dtype and out.shape == t['z_tr'].shape
    ref = oracle.contextualize(case['z_tr'], case['v'], case['z_tl'], case['bias'],
                               case['valid'], **kw)
    assert norm_rel_err(to_numpy(out), ref) <= TOL[case['dtype']]


def test_custom_op_traces_with_fake_tensors():
    from torch.fx.experimental.proxy_tensor import make_fx

    def fn(x):
        return ops.contextualize(x, None, x, None, None, 1e-6, 1e-12, False, True, 0)

    graph = make_fx(fn, tracing_mode='fake')(torch.empty(2, 35, 37))
    calls = [n for n in graph.graph.nodes if 'avey_b200.contextualize' in str(n.target)]
    assert len(calls) == 1


def test_dynamo_fullgraph_over_the_custom_op_without_cuda():
    from torch._subclasses.fake_tensor import FakeTensorMode

    def fn(z):
        return avey_b(z, backend='cuda') if z.is_cuda else ops.contextualize(
            z, None, None, None, None, 1e-6, 1e-12, False, True, 0)

    compiled = torch.compile(fn, backend='eager', fullgraph=True, dynamic=True)
    with FakeTensorMode():
        for shape in ((1, 5, 7), (2, 35, 40)):
            z = torch.empty(*shape)
            result = compiled(z)
            assert result.shape == z.shape and result.dtype == z.dtype


def test_oracle_is_not_imported_by_the_product_package():
    code = ('import sys, avey_kernel_b200, avey_kernel_b200.ops, avey_kernel_b200.eager; '
            'print("oracle" in sys.modules)')
    out = subprocess.run([sys.executable, '-c', code], capture_output=True, text=True,
                         cwd=str(ROOT))
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == 'False'
