"""The 8-row CUDA-core kernel for small fp32 problems (small_kernel.cuh) on a
B200, against the oracle.

AUTO runs small fp32 inputs (contexts up to 512, features a multiple of 32
up to 256, up to 4 waves of query tiles of 8 rows, 2 at 128 tokens or fewer)
on this kernel, config 1 among them; each tile runs on a CTA pair that splits
its keys. Bound: the north-star fp32 bound norm-wise (1e-4), and 1e-5
elementwise (rtol, with an atol of 1e-5 of the largest output). Covered:
Avey (causal, learned V, bias, every activation) and Avey-B (bidirectional,
signed row-sum divide), both key-block sizes (128 keys for rows up to 512
bytes, 64 above), one to four blocks with the double buffering wrapping,
contexts that are not a multiple of the 8-row tile, byte masks and prefix
lengths with NaN in the padding, head/tail views of one buffer, and one
launch per call.
"""

import numpy as np
import pytest
import torch

import oracle
from avey_kernel_b200 import _native, ops
from helpers import TOL, norm_rel_err, to_numpy

pytestmark = pytest.mark.gpu
DEV = 'cuda'
ACTS = ['identity', 'relu', 'relu2', 'silu', 'gelu']


@pytest.fixture(autouse=True)
def _device_status_clean():
    _native.device_status(clear=True)
    yield
    assert _native.device_status(clear=True) == 0


def _inputs(b, n, d, seed, signed_tail=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, n, 2 * d, generator=g)
    if not signed_tail:  # Avey-B: keep the signed row sums away from -eps
        x[..., d:] = x[..., d:].abs()
    x = x.to(DEV)
    v = (torch.randn(n, n, generator=g) * 0.05).to(DEV)
    bias = (torch.randn(d, generator=g) * 0.1).to(DEV)
    lengths = torch.randint(1, n + 1, (b,), generator=g)
    valid = (torch.arange(n)[None, :] < lengths[:, None]).to(DEV)
    return x, v, bias, valid


def _check(y, ref):
    y = to_numpy(y)
    assert np.isfinite(y).all()
    assert norm_rel_err(y, ref) <= TOL['float32'], norm_rel_err(y, ref)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * max(1.0, float(np.abs(ref).max())))


def _small_plan(tail, v, head, bias, valid, causal, normalize):
    plan = ops.plan(tail, v, head, bias, valid, causal=causal, normalize=normalize)
    assert plan.kernel == _native.KERNEL_SIMT and plan.reason == _native.REASON_SMALL
    return plan


@pytest.mark.parametrize('act', ACTS)
@pytest.mark.parametrize('b,n,d', [(2, 256, 128), (3, 100, 64), (1, 512, 128), (1, 300, 256),
                                   (4, 7, 32), (1, 333, 96)])
def test_avey_causal(b, n, d, act):
    x, v, bias, _ = _inputs(b, n, d, seed=n + d)
    head, tail = x[..., :d], x[..., d:]
    _small_plan(tail, v, head, bias, None, True, False)
    before = _native.launch_count()
    y = ops.contextualize(tail, v, head, bias, None, 1e-6, 1e-12, True, False,
                          _native.ACTIVATION_IDS[act])
    torch.cuda.synchronize()
    assert _native.launch_count() == before + 1
    ref = oracle.avey(to_numpy(tail), to_numpy(v), z_tl=to_numpy(head), bias=to_numpy(bias),
                      activation=act)
    _check(y, ref)


@pytest.mark.parametrize('act', ['identity', 'gelu'])
@pytest.mark.parametrize('b,n,d', [(2, 256, 128), (2, 200, 256), (2, 400, 64), (5, 9, 32)])
def test_avey_b_with_ragged_padding(b, n, d, act):
    x, _, _, valid = _inputs(b, n, d, seed=3 * n + d, signed_tail=False)
    head, tail = x[..., :d], x[..., d:]
    tail[~valid] = float('nan')  # padding is never read
    _small_plan(tail, None, head, None, valid, False, True)
    y = ops.contextualize(tail, None, head, None, valid, 1e-6, 1e-12, False, True,
                          _native.ACTIVATION_IDS[act])
    torch.cuda.synchronize()
    ok = to_numpy(valid.float()) > 0
    ref = oracle.avey_b(np.nan_to_num(to_numpy(tail)), z_tl=to_numpy(head), valid=ok,
                        activation=act)
    _check(y, ref)
    assert (to_numpy(y)[~ok] == 0).all()


def test_avey_causal_with_mask_and_lengths_agree():
    """The byte mask and the prefix-length form of the same padding give the
    same bits (the C ABI's lengths field)."""
    b, n, d = 3, 256, 128
    x, v, bias, valid = _inputs(b, n, d, seed=77)
    head, tail = x[..., :d], x[..., d:]
    _small_plan(tail, v, head, bias, valid, True, False)
    y = ops.contextualize(tail, v, head, bias, valid, 1e-6, 1e-12, True, False, 3)
    ok = to_numpy(valid.float()) > 0
    ref = oracle.avey(to_numpy(tail), to_numpy(v), z_tl=to_numpy(head), bias=to_numpy(bias),
                      valid=ok, activation='silu')
    _check(y, ref)
    out = torch.empty_like(tail)
    params = ops.build_params(tail, v, head, bias, None, out, eps=1e-6, norm_eps=1e-12,
                              causal=True, normalize=False, activation_id=3)
    lengths = valid.sum(dim=1).to(torch.int32)
    params.lengths = lengths.data_ptr()
    _native.forward(params, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(out, y)


@pytest.mark.parametrize('b,n,d', [(2, 256, 128), (2, 96, 256)])
def test_matches_the_3xtf32_pair_and_the_two_phase_kernel(b, n, d):
    """AUTO (this kernel), the forced 3xTF32 pair and the forced two-phase
    CUDA-core kernel agree within the fp32 bound."""
    x, v, _, _ = _inputs(b, n, d, seed=5)
    head, tail = x[..., :d], x[..., d:]
    ys = [ops.contextualize(tail, v, head, None, None, 1e-6, 1e-12, True, False, 0, k)
          for k in (_native.KERNEL_AUTO, _native.KERNEL_TCGEN05, _native.KERNEL_SIMT)]
    torch.cuda.synchronize()
    for y in ys[1:]:
        assert norm_rel_err(to_numpy(ys[0]), to_numpy(y)) <= TOL['float32']


@pytest.mark.parametrize('op', ['avey', 'avey_b'])
def test_rows_that_are_all_padding(op):
    """A batch row of length 0 beside full and short ones: its CTA pairs have no
    key block (they still take part in the pair's combine) and its output is
    zero; the other rows match the oracle."""
    b, n, d = 3, 136, 64
    x, v, bias, _ = _inputs(b, n, d, seed=91, signed_tail=op == 'avey')
    head, tail = x[..., :d], x[..., d:]
    lengths = torch.tensor([0, n, 37])
    valid = (torch.arange(n)[None, :] < lengths[:, None]).to(DEV)
    tail[~valid] = float('nan')
    causal, normalize = op == 'avey', op == 'avey_b'
    _small_plan(tail, v if causal else None, head, bias, valid, causal, normalize)
    y = ops.contextualize(tail, v if causal else None, head, bias, valid, 1e-6, 1e-12, causal,
                          normalize, _native.ACTIVATION_IDS['silu'])
    torch.cuda.synchronize()
    ok = to_numpy(valid.float()) > 0
    zt = np.nan_to_num(to_numpy(tail))
    if causal:
        ref = oracle.avey(zt, to_numpy(v), z_tl=to_numpy(head), bias=to_numpy(bias), valid=ok,
                          activation='silu')
    else:
        ref = oracle.avey_b(zt, z_tl=to_numpy(head), bias=to_numpy(bias), valid=ok,
                            activation='silu')
    out = to_numpy(y)
    assert np.isfinite(out).all()
    assert (out[0] == 0).all() and (out[~ok] == 0).all()
    for r in (1, 2):
        _check(y[r:r + 1], ref[r:r + 1])
