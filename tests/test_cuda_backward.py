"""The native backward (``avey_kernel_b200/backward.py``) on a B200.

Gradients of ``avey`` / ``avey_b`` through torch autograd on CUDA tensors,
which runs the C-ABI backward steps and library GEMMs, compared with

* the gradient oracle (``oracle/backward.py``, fp64) and the reference's own
  gradients (``tests/golden/grad_golden.npz``) on every gradient golden case;
* torch.autograd.gradcheck in fp64 (the reference's test_contextualizer.py:41-47);
* the oracle at tensor-core sizes (bf16, causal and bidirectional, masks).

Tolerances, norm-wise against the fp64 oracle: fp64 1e-9, fp32 1e-4, fp16 /
bf16 2e-2 (the forward's bounds). Gradients are also bitwise reproducible.
"""

import numpy as np
import pytest
import torch

from avey_kernel_b200 import _native, avey, avey_b
from fixtures import GRAD_FIELDS, grad_to_torch, load_grad_cases, oracle_kwargs
from oracle.backward import contextualize_backward

pytestmark = pytest.mark.gpu
DEV = 'cuda'
TOL = {torch.float64: 1e-9, torch.float32: 1e-4, torch.float16: 2e-2, torch.bfloat16: 2e-2}
GRAD_CASES = load_grad_cases()


def normwise(got, ref):
    scale = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got - ref))) / (scale if scale > 0 else 1.0)


def forward(op, t, kw, backend='cuda'):
    if op == 'avey':
        return avey(t['z_tr'], t['v'], z_tl=t['z_tl'], bias=t['bias'], valid=t['valid'],
                    causal=kw['causal'], activation=kw['activation'], backend=backend)
    return avey_b(t['z_tr'], z_tl=t['z_tl'], bias=t['bias'], valid=t['valid'], eps=kw['eps'],
                  activation=kw['activation'], backend=backend)


def native_grads(op, t, kw, grad_out):
    leaves = {}
    for f in GRAD_FIELDS:
        leaves[f] = None if t[f] is None else t[f].detach().clone().requires_grad_(True)
    tt = dict(t, **leaves)
    out = forward(op, tt, kw)
    out.backward(grad_out)
    return [None if leaves[f] is None else leaves[f].grad for f in GRAD_FIELDS]


def np64(t):
    return None if t is None else t.detach().double().cpu().numpy()


@pytest.fixture(autouse=True)
def _device_status_clean():
    _native.device_status(clear=True)
    yield
    assert _native.device_status(clear=True) == 0


@pytest.mark.parametrize('case', GRAD_CASES, ids=[c['name'] for c in GRAD_CASES])
def test_golden_gradients(case):
    t = grad_to_torch(case, DEV)
    kw = oracle_kwargs(case)
    before = _native.launch_count()
    grads = native_grads(case['op'], t, kw, t['grad_out'])
    torch.cuda.synchronize()
    assert _native.launch_count() > before + 1, 'native forward and backward steps did not launch'
    ref = contextualize_backward(case['z_tr'], case['v'], case['z_tl'], case['bias'],
                                 case['valid'], case['grad_out'], **kw)
    tol = TOL[t['z_tr'].dtype]
    for field, got, want, golden in zip(GRAD_FIELDS, grads, ref, [case['d_' + f] for f in GRAD_FIELDS]):
        if want is None:
            assert got is None, field
            continue
        assert got.dtype == t[field].dtype and got.shape == t[field].shape, field
        g = np64(got)
        assert np.isfinite(g).all(), field
        assert normwise(g, want) <= tol, (field, normwise(g, want))
        assert normwise(g, golden.astype(np.float64)) <= max(tol, 2e-2 if tol > 1e-4 else 1e-4), field


def test_gradcheck_fp64_like_the_reference():
    g = torch.Generator().manual_seed(0)
    z = torch.rand(1, 3, 2, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    v = torch.rand(3, 3, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    assert torch.autograd.gradcheck(lambda x, w: avey(x, w), (z, v))
    assert torch.autograd.gradcheck(lambda x: avey_b(x), (z,))
    z = torch.randn(2, 37, 9, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    zl = torch.randn(2, 37, 9, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    b = torch.randn(9, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    w = torch.randn(37, 37, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    valid = (torch.rand(2, 37, generator=g) > 0.2).to(DEV)
    assert torch.autograd.gradcheck(
        lambda x, ww, gl, bb: avey(x, ww, z_tl=gl, bias=bb, valid=valid, activation='gelu'),
        (z, w, zl, b))
    assert torch.autograd.gradcheck(
        lambda x, gl, bb: avey_b(x, z_tl=gl, bias=bb, valid=valid, eps=0.5, activation='silu'),
        (z, zl, b))


def test_nan_padding_cannot_contaminate_gradients():
    for normalized in (False, True):
        z = torch.tensor([[[1., 2.], [3., 4.], [float('nan'), float('nan')]]], device=DEV,
                         requires_grad=True)
        zl = torch.tensor([[[1., 1.], [1., 1.], [float('nan'), float('nan')]]], device=DEV,
                          requires_grad=True)
        valid = torch.tensor([[True, True, False]], device=DEV)
        out = (avey_b(z, z_tl=zl, valid=valid) if normalized
               else avey(z, torch.ones(3, 3, device=DEV), z_tl=zl, valid=valid))
        out.sum().backward()
        assert torch.isfinite(z.grad).all() and torch.isfinite(zl.grad).all()
        assert (z.grad[:, -1] == 0).all() and (zl.grad[:, -1] == 0).all()


@pytest.mark.parametrize('op,b,n,d', [('avey', 2, 256, 192), ('avey_b', 3, 384, 128),
                                      ('avey', 1, 640, 96),
                                      # three feature slots per epilogue pass: one pass, two passes
                                      ('avey', 1, 256, 520), ('avey_b', 2, 128, 1040)])
def test_tensor_core_sizes_bf16(op, b, n, d):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(b, n, 2 * d, generator=g).to(torch.bfloat16)
    t = dict(z_tr=x[..., d:].to(DEV), z_tl=x[..., :d].to(DEV), bias=None, valid=None,
             v=(torch.randn(n, n, generator=g) * 0.02).to(torch.bfloat16).to(DEV) if op == 'avey' else None)
    if op == 'avey_b':
        lengths = torch.randint(n // 4, n + 1, (b,), generator=g)
        t['valid'] = (torch.arange(n)[None, :] < lengths[:, None]).to(DEV)
    else:
        t['bias'] = (torch.randn(d, generator=g) * 0.01).to(torch.bfloat16).to(DEV)
    kw = dict(causal=op == 'avey', activation='identity', eps=1e-6, norm_eps=1e-12,
              normalize=op == 'avey_b')
    go = torch.randn(b, n, d, generator=g).to(torch.bfloat16).to(DEV)
    grads = native_grads(op, t, kw, go)
    ref = contextualize_backward(np64(t['z_tr']), np64(t['v']), np64(t['z_tl']), np64(t['bias']),
                                 None if t['valid'] is None else t['valid'].cpu().numpy(),
                                 np64(go), **kw)
    for field, got, want in zip(GRAD_FIELDS, grads, ref):
        if want is None:
            continue
        assert normwise(np64(got), want) <= 2e-2, (field, normwise(np64(got), want))


def test_gradients_are_bitwise_reproducible_and_subsets_match():
    g = torch.Generator().manual_seed(5)
    z = torch.randn(3, 130, 64, generator=g).to(DEV)
    zl = torch.randn(3, 130, 64, generator=g).to(DEV)
    w = (torch.randn(130, 130, generator=g) * 0.1).to(DEV)
    b = torch.randn(64, generator=g).to(DEV)
    go = torch.randn(3, 130, 64, generator=g).to(DEV)

    def run(**req):
        leaves = [t.clone().requires_grad_(req.get(k, True))
                  for k, t in (('z', z), ('w', w), ('zl', zl), ('b', b))]
        avey(leaves[0], leaves[1], z_tl=leaves[2], bias=leaves[3], activation='silu').backward(go)
        return [None if t.grad is None else t.grad.clone() for t in leaves]

    first, second = run(), run()
    for a, c in zip(first, second):
        assert torch.equal(a, c)
    only_gate = run(z=False, w=False, b=False)
    assert only_gate[0] is None and only_gate[1] is None and only_gate[3] is None
    assert torch.equal(only_gate[2], first[2])
    only_v = run(z=False, zl=False, b=False)
    assert torch.equal(only_v[1], first[1])


def test_custom_ops_pass_opcheck():
    from avey_kernel_b200 import backward, ops
    g = torch.Generator().manual_seed(1)
    z = torch.randn(2, 20, 16, generator=g).to(DEV).requires_grad_(True)
    w = torch.randn(20, 20, generator=g).to(DEV).requires_grad_(True)
    zl = torch.randn(2, 20, 16, generator=g).to(DEV)
    torch.library.opcheck(ops.contextualize, (z, w, zl, None, None, 1e-6, 1e-12, True, False, 3, 0))
    go = torch.randn(2, 20, 16, generator=g).to(DEV)
    torch.library.opcheck(backward.contextualize_backward,
                          (z.detach(), w.detach(), zl, None, None, go, 1e-6, 1e-12, True, False, 3,
                           [True, True, True, False]))


@pytest.mark.parametrize('d', [48, 520])  # two and three feature slots per epilogue pass
@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16, torch.float16])
def test_vector_and_scalar_steps_agree(dtype, d):
    # The same values once in 16-byte aligned rows (vector steps) and once
    # shifted by one element (scalar steps).
    g = torch.Generator().manual_seed(9)
    b, n = 2, 64
    base = torch.randn(b, n, 2 * d + 1, generator=g).to(dtype).to(DEV)
    w = (torch.randn(n, n, generator=g) * 0.1).to(dtype).to(DEV)
    go = torch.randn(b, n, d, generator=g).to(dtype).to(DEV)
    aligned = base[..., :2 * d].clone()
    shifted = base[..., 1:].clone()
    shifted.copy_(aligned)  # same values, rows start 2 or 4 bytes past 16
    grads = []
    for x in (aligned, shifted):
        xl = x.detach().requires_grad_(True)
        wl = w.clone().requires_grad_(True)
        out = avey(xl[..., d:], wl, z_tl=xl[..., :d], activation='gelu')
        grads.append(torch.autograd.grad(out, (xl, wl), go))
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for a, c in zip(*grads):
        assert normwise(np64(a), np64(c)) <= tol


@pytest.mark.parametrize('op', ['avey', 'avey_b'])
def test_packed_head_tail_views_take_one_gradient(op):
    # z_tl / z_tr as the halves of one [B, C, 2d'] tensor: the packed op gives
    # x one gradient; it must equal the gradients of separate tensors.
    g = torch.Generator().manual_seed(21)
    b, n, d = 2, 200, 96
    x0 = torch.randn(b, n, 2 * d, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(n, n, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(d, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    go = torch.randn(b, n, d, generator=g).to(torch.bfloat16).to(DEV)

    def run(zt, zl, bb):
        if op == 'avey':
            return avey(zt, w, z_tl=zl, bias=bb, activation='relu')
        return avey_b(zt, z_tl=zl, bias=bb, eps=0.5, activation='relu')

    x = x0.clone().requires_grad_(True)
    b1 = bias.clone().requires_grad_(True)
    out = run(x[..., d:], x[..., :d], b1)
    assert 'contextualize_packed' in out.grad_fn.name()
    gx, gb = torch.autograd.grad(out, (x, b1), go)
    zt = x0[..., d:].clone().requires_grad_(True)
    zl = x0[..., :d].clone().requires_grad_(True)
    b2 = bias.clone().requires_grad_(True)
    out2 = run(zt, zl, b2)
    assert 'contextualize_packed' not in out2.grad_fn.name()
    assert torch.equal(out, out2)
    gzt, gzl, gb2 = torch.autograd.grad(out2, (zt, zl, b2), go)
    assert torch.equal(gx[..., d:], gzt) and torch.equal(gx[..., :d], gzl)
    assert torch.equal(gb, gb2)


def test_packed_custom_ops_pass_opcheck():
    from avey_kernel_b200 import backward, ops
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 24, 32, generator=g).to(DEV).requires_grad_(True)
    w = torch.randn(24, 24, generator=g).to(DEV).requires_grad_(True)
    torch.library.opcheck(ops.contextualize_packed, (x, w, None, None, 1e-6, 1e-12, True, False, 4))
    go = torch.randn(2, 24, 16, generator=g).to(DEV)
    torch.library.opcheck(backward.contextualize_packed_backward,
                          (x.detach(), w.detach(), None, None, go, 1e-6, 1e-12, True, False, 4,
                           [True, True, False]))


def test_training_step_replays_from_a_cuda_graph():
    # Forward + backward captured once and replayed: the same gradients as eager.
    g = torch.Generator().manual_seed(8)
    b, n, d = 2, 128, 64
    x = torch.randn(b, n, 2 * d, generator=g).to(torch.bfloat16).to(DEV).requires_grad_(True)
    w = (torch.randn(n, n, generator=g) * 0.05).to(torch.bfloat16).to(DEV).requires_grad_(True)
    go = torch.randn(b, n, d, generator=g).to(torch.bfloat16).to(DEV)

    def step():
        out = avey(x[..., d:], w, z_tl=x[..., :d], activation='gelu')
        return torch.autograd.grad(out, (x, w), go)

    eager = step()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step()
    graph.replay()
    torch.cuda.synchronize()
    for a, c in zip(eager, captured):
        assert torch.equal(a, c)
