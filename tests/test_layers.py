"""The layers on either side of the contextualizer (``avey_kernel_b200.layers``):
the enricher (with the tail's row sums of squares from its epilogue), the
enricher + contextualizer pipeline (``avey_fwd_presummed_v1``, no row-norm
pre-pass) and the static layers.

References: fp64 PyTorch products of the same 16-bit operands for the GEMM
layers (bf16 / f16 rounding of the stored output, 1e-2 of the output scale),
and the NumPy oracle of the reference's ``_reference`` for the contextualizer
step (2e-2 norm-wise, the forward's bound). CPU inputs take plain PyTorch.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from avey_kernel_b200 import _native, layers, ops
from helpers import TOL, norm_rel_err, to_numpy

DEV = 'cuda'
ACTS = ['identity', 'relu', 'relu2', 'silu', 'gelu']


def torch_act(y, activation):
    return {'identity': lambda t: t, 'relu': torch.relu, 'relu2': lambda t: torch.relu(t) ** 2,
            'silu': F.silu, 'gelu': lambda t: F.gelu(t, approximate='tanh')}[activation](y)


def within(got, ref, frac=1e-2):
    scale = float(ref.abs().max())
    return float((got.double() - ref).abs().max()) <= frac * max(scale, 1e-30)


# ---------------------------------------------------------------- CPU (plain PyTorch)

def test_cpu_paths_are_plain_pytorch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 16, 24, generator=g)
    w = torch.randn(32, 24, generator=g)
    b = torch.randn(32, generator=g)
    e, sums = layers.enrich(x, w, b, activation='silu', tail_sums=True)
    assert sums is None
    torch.testing.assert_close(e, F.silu(F.linear(x, w, b)))
    gate = torch.randn(2, 16, 32, generator=g)
    torch.testing.assert_close(layers.static_linear(x, w, b, activation='relu', gate=gate),
                               torch.relu(F.linear(x, w, b)) * gate)
    wm = torch.randn(16, 16, generator=g)
    torch.testing.assert_close(layers.static_mix(x, wm, causal=True), torch.matmul(wm.tril(), x))
    out = layers.avey_enriched(x, w, wm, enrich_activation='relu')
    ee = torch.relu(F.linear(x, w))
    torch.testing.assert_close(out, ops.avey(ee[..., 16:], wm, z_tl=ee[..., :16]))


@pytest.mark.parametrize('call,match', [
    (lambda: layers.enrich(torch.randn(2, 3, 4), torch.randn(6, 5)), 'weight'),
    (lambda: layers.enrich(torch.randn(2, 3, 4), torch.randn(5, 4)), 'weight'),
    (lambda: layers.static_linear(torch.randn(2, 3, 4), torch.randn(6, 4), torch.randn(5)), 'bias'),
    (lambda: layers.static_mix(torch.randn(2, 3, 4), torch.randn(4, 4)), 'weight'),
    (lambda: layers.static_linear(torch.randn(2, 3, 4), torch.randn(6, 4), activation='tanh'),
     'activation'),
])
def test_contract_errors(call, match):
    with pytest.raises(ValueError, match=match):
        call()


# ---------------------------------------------------------------- GPU (native)

@pytest.fixture
def clean_status():
    _native.device_status(clear=True)
    yield
    assert _native.device_status(clear=True) == 0


@pytest.mark.gpu
@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('act', ACTS)
def test_enrich_and_tail_sums(dtype, act, clean_status):
    g = torch.Generator().manual_seed(ACTS.index(act))
    bt, c, d_in, d = 3, 200, 192, 256
    x = torch.randn(bt, c, d_in, generator=g).to(dtype).to(DEV)
    w = (torch.randn(2 * d, d_in, generator=g) * d_in ** -0.5).to(dtype).to(DEV)
    b = (torch.randn(2 * d, generator=g) * 0.1).to(dtype).to(DEV)
    e, sums = layers.enrich(x, w, b, activation=act, tail_sums=True)
    torch.cuda.synchronize()
    ref = torch_act(F.linear(x.double(), w.double(), b.double()), act)
    assert within(e, ref)
    assert sums.shape == (d // 128, bt * c)
    tail2 = e.float()[..., d:] ** 2
    for p in range(d // 128):
        torch.testing.assert_close(sums[p], tail2[..., 128 * p:128 * p + 128].sum(-1).reshape(-1),
                                   rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize('op', ['avey', 'avey_b'])
def test_enriched_pipeline_matches_oracle(op, clean_status):
    """Enricher + contextualizer with the row norms from the enricher's
    epilogue: against the oracle on the enriched tensor, and against the
    contextualizer with its own pre-pass on the same tensor."""
    g = torch.Generator().manual_seed(7)
    bt, c, d_in, d = 4, 512, 256, 384
    x = torch.randn(bt, c, d_in, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(2 * d, d_in, generator=g) * d_in ** -0.5).to(torch.bfloat16).to(DEV)
    be = (torch.randn(2 * d, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    bias = (torch.randn(d, generator=g) * 0.01).to(torch.bfloat16).to(DEV)
    v = (torch.randn(c, c, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    lengths = torch.randint(c // 4, c + 1, (bt,), generator=g)
    valid = (torch.arange(c)[None, :] < lengths[:, None]).to(DEV)
    e, _ = layers.enrich(x, w, be, activation='relu')
    head, tail = e[..., :d], e[..., d:]
    before = _native.launch_count()
    if op == 'avey':
        got = layers.avey_enriched(x, w, v, enrich_bias=be, enrich_activation='relu', bias=bias,
                                   activation='silu')
        plain = ops.avey(tail, v, z_tl=head, bias=bias, activation='silu')
        ref = oracle.avey(to_numpy(tail), to_numpy(v), z_tl=to_numpy(head), bias=to_numpy(bias),
                          activation='silu')
    else:
        got = layers.avey_b_enriched(x, w, enrich_bias=be, enrich_activation='relu', valid=valid,
                                     eps=0.5, activation='gelu')
        plain = ops.avey_b(tail, z_tl=head, valid=valid, eps=0.5, activation='gelu')
        ref = oracle.avey_b(to_numpy(tail), z_tl=to_numpy(head), valid=to_numpy(valid), eps=0.5,
                            activation='gelu')
    torch.cuda.synchronize()
    # enricher GEMM + plane sums + fused kernel (no pass over z_tr), then the plain call's
    # fused kernel (which sums the rows' squares itself)
    assert _native.launch_count() == before + 3 + 1
    assert norm_rel_err(to_numpy(got), ref) <= TOL['bfloat16']
    assert norm_rel_err(to_numpy(got), to_numpy(plain)) <= 2e-3


@pytest.mark.gpu
@pytest.mark.parametrize('act', ['identity', 'gelu'])
@pytest.mark.parametrize('with_gate', [False, True])
def test_static_linear(act, with_gate, clean_status):
    g = torch.Generator().manual_seed(3)
    bt, c, d_in, d_out = 2, 300, 384, 520
    x = torch.randn(bt, c, d_in, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(d_out, d_in, generator=g) * d_in ** -0.5).to(torch.bfloat16).to(DEV)
    b = (torch.randn(d_out, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    gate = torch.randn(bt, c, d_out, generator=g).to(torch.bfloat16).to(DEV) if with_gate else None
    got = layers.static_linear(x, w, b, activation=act, gate=gate)
    ref = torch_act(F.linear(x.double(), w.double(), b.double()), act)
    if with_gate:
        ref = ref * gate.double()
    assert within(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize('causal', [False, True])
def test_static_mix(causal, clean_status):
    g = torch.Generator().manual_seed(4)
    bt, c, d = 3, 512, 384
    z = torch.randn(bt, c, d, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(c, c, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    b = (torch.randn(d, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    gate = torch.randn(bt, c, d, generator=g).to(torch.bfloat16).to(DEV)
    got = layers.static_mix(z, w, bias=b, activation='silu', gate=gate, causal=causal)
    wr = w.double().tril() if causal else w.double()
    ref = F.silu(torch.matmul(wr, z.double()) + b.double()) * gate.double()
    assert within(got, ref)


@pytest.mark.gpu
def test_enriched_pipeline_with_autograd():
    """Inputs that require grad: the enricher runs in PyTorch, the
    contextualizer natively with its native backward."""
    g = torch.Generator().manual_seed(9)
    bt, c, d_in, d = 2, 256, 128, 128
    x = torch.randn(bt, c, d_in, generator=g).to(torch.bfloat16).to(DEV).requires_grad_(True)
    w = (torch.randn(2 * d, d_in, generator=g) * d_in ** -0.5).to(torch.bfloat16).to(DEV)
    w.requires_grad_(True)
    v = (torch.randn(c, c, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    out = layers.avey_enriched(x, w, v, enrich_activation='relu')
    out.float().square().sum().backward()
    xe, we = x.detach().double().cpu().requires_grad_(True), w.detach().double().cpu().requires_grad_(True)
    e = torch.relu(F.linear(xe, we))
    ref = ops.avey(e[..., d:], v.double().cpu(), z_tl=e[..., :d], backend='torch')
    (ref.square().sum()).backward()
    assert norm_rel_err(to_numpy(out), to_numpy(ref)) <= TOL['bfloat16']
    assert norm_rel_err(to_numpy(x.grad), to_numpy(xe.grad)) <= 5e-2
    assert norm_rel_err(to_numpy(w.grad), to_numpy(we.grad)) <= 5e-2


@pytest.mark.gpu
def test_enriched_pipeline_long_context_and_fallbacks(clean_status):
    """The pre-summed contextualizer on the long-context path (640 tokens: the
    plane sums feed the G/P and P.Z kernels), and a width whose tail is not a
    whole number of 128-column planes (no sums: the contextualizer runs its own
    pre-pass)."""
    g = torch.Generator().manual_seed(11)
    for c, d, sums_expected in ((640, 256, True), (256, 200, False)):
        x = torch.randn(2, c, 128, generator=g).to(torch.bfloat16).to(DEV)
        w = (torch.randn(2 * d, 128, generator=g) * 128 ** -0.5).to(torch.bfloat16).to(DEV)
        v = (torch.randn(c, c, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
        e, sums = layers.enrich(x, w, activation='silu', tail_sums=True)
        assert (sums is not None) == sums_expected
        got = layers.avey_enriched(x, w, v, enrich_activation='silu', activation='relu')
        head, tail = e[..., :d], e[..., d:]
        ref = oracle.avey(to_numpy(tail), to_numpy(v), z_tl=to_numpy(head), activation='relu')
        plain = ops.avey(tail, v, z_tl=head, activation='relu')
        torch.cuda.synchronize()
        assert norm_rel_err(to_numpy(got), ref) <= TOL['bfloat16']
        assert norm_rel_err(to_numpy(got), to_numpy(plain)) <= 2e-3


@pytest.mark.gpu
def test_presummed_entry_point_matches_the_plain_one(clean_status):
    """avey_fwd_presummed_v1 through the C ABI with sums computed here in two
    planes, against avey_fwd_v1 (its own pre-pass) on the same tensors: the
    same kernels up to the summation order of the row norms."""
    g = torch.Generator().manual_seed(12)
    x = torch.randn(3, 512, 2 * 256, generator=g).to(torch.bfloat16).to(DEV)
    head, tail = x[..., :256], x[..., 256:]
    tf = tail.float()
    planes = torch.stack([(tf[..., :128] ** 2).sum(-1).reshape(-1),
                          (tf[..., 128:] ** 2).sum(-1).reshape(-1)]).contiguous()
    outs = []
    for presummed in (False, True):
        out = torch.empty(tail.shape, dtype=tail.dtype, device=DEV)
        p = ops.build_params(tail, None, head, None, None, out, eps=0.5, norm_eps=1e-12,
                             causal=False, normalize=True, activation_id=4)
        # avey_fwd_v1 needs none here (the fused kernel sums the rows); the
        # pre-summed entry combines the planes into one float per row.
        n = max(_native.workspace_size(p), 4 * 3 * 512) if presummed else _native.workspace_size(p)
        ws = torch.empty(max(n, 1), dtype=torch.uint8, device=DEV)
        p.workspace, p.workspace_bytes = ws.data_ptr(), n
        stream = torch.cuda.current_stream().cuda_stream
        if presummed:
            _native.forward_presummed(p, planes.data_ptr(), 2, stream)
        else:
            _native.forward(p, stream)
        torch.cuda.synchronize()
        outs.append(out)
    # The two differ only in the summation order of the row norms (last bits of
    # rinv), which can move a bf16 rounding of P by one unit (2^-9 relative).
    assert norm_rel_err(to_numpy(outs[1]), to_numpy(outs[0])) <= 5e-3
    ref = oracle.avey_b(to_numpy(tail), z_tl=to_numpy(head), eps=0.5, activation='gelu')
    assert norm_rel_err(to_numpy(outs[1]), ref) <= TOL['bfloat16']
