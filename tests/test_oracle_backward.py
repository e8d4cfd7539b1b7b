"""The gradient oracle (``oracle/backward.py``), pinned on CPU.

1. Against the reference's own gradients: torch autograd through
   ``avey_kernels/ops.py::_reference``, stored by
   ``tests/golden/make_grad_golden.py`` (fp64 cases to 1e-10; fp32 cases to
   1e-5; 16-bit cases, whose reference gradients are rounded to the input
   dtype, to 2e-2; all norm-wise).
2. Against central finite differences of the forward oracle (fp64).
3. NaN padding never reaches a gradient, and padded rows get zero gradient
   (the reference's tests/test_contextualizer.py:49-62).
"""

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
import oracle  # noqa: E402
from oracle.backward import contextualize_backward  # noqa: E402
from fixtures import GRAD_FIELDS, load_grad_cases, oracle_kwargs  # noqa: E402

TOL = {'float64': 1e-10, 'float32': 1e-5, 'float16': 2e-2, 'bfloat16': 2e-2}


def oracle_grads(case, accum=np.float64):
    return contextualize_backward(case['z_tr'], case['v'], case['z_tl'], case['bias'],
                                  case['valid'], case['grad_out'], accum=accum,
                                  **oracle_kwargs(case))


def normwise(got, ref):
    scale = np.max(np.abs(ref))
    return float(np.max(np.abs(got - ref)) / (scale if scale > 0 else 1.0))


@pytest.mark.parametrize('case', load_grad_cases(), ids=[c['name'] for c in load_grad_cases()])
def test_oracle_matches_reference_gradients(case):
    grads = oracle_grads(case)
    for field, got in zip(GRAD_FIELDS, grads):
        ref = case['d_' + field]
        if ref is None:
            assert got is None or case[field] is None, field
            continue
        assert np.isfinite(got).all(), field
        assert normwise(got, ref.astype(np.float64)) <= TOL[case['dtype']], field


@pytest.mark.parametrize('normalize,causal,act', [(False, True, 'identity'), (False, False, 'gelu'),
                                                  (True, False, 'silu'), (True, False, 'relu2')])
def test_oracle_matches_finite_differences(normalize, causal, act):
    rng = np.random.default_rng(3)
    b, c, d = 2, 6, 5
    z = rng.standard_normal((b, c, d))
    v = None if normalize else rng.standard_normal((c, c))
    zl = rng.standard_normal((b, c, d))
    bias = rng.standard_normal(d)
    valid = np.ones((b, c), dtype=bool)
    valid[1, 2] = False
    go = rng.standard_normal((b, c, d))
    kw = dict(eps=0.5 if normalize else 1e-6, norm_eps=1e-12, causal=causal,
              normalize=normalize, activation=act)
    grads = contextualize_backward(z, v, zl, bias, valid, go, **kw)

    def loss(zz, vv, ll, bb):
        return float((oracle.contextualize(zz, vv, ll, bb, valid, **kw) * go).sum())

    h = 1e-6
    args = [z, v, zl, bias]
    for k, g in enumerate(grads):
        if args[k] is None:
            continue
        flat = args[k].reshape(-1)
        num = np.zeros_like(flat)
        for idx in range(flat.size):
            old = flat[idx]
            flat[idx] = old + h
            up = loss(*args)
            flat[idx] = old - h
            dn = loss(*args)
            flat[idx] = old
            num[idx] = (up - dn) / (2 * h)
        np.testing.assert_allclose(g.reshape(-1), num, rtol=1e-5, atol=1e-6)


def test_nan_padding_gives_zero_gradients_on_padded_rows():
    z = np.array([[[1., 2.], [3., 4.], [np.nan, np.nan]]])
    zl = np.array([[[1., 1.], [1., 1.], [np.nan, np.nan]]])
    valid = np.array([[True, True, False]])
    go = np.ones_like(z)
    for normalize in (False, True):
        gz, _, gzl, _ = contextualize_backward(
            z, None if normalize else np.ones((3, 3)), zl, None, valid, go, eps=1e-6,
            norm_eps=1e-12, causal=not normalize, normalize=normalize)
        assert np.isfinite(gz).all() and np.isfinite(gzl).all()
        assert (gz[:, -1] == 0).all() and (gzl[:, -1] == 0).all()
