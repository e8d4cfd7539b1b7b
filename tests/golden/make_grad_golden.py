"""Generate the gradient golden vectors ``tests/golden/grad_golden.npz`` +
``grad_cases.json``.

Each case holds seeded inputs, a seeded upstream gradient ``grad_out`` and the
gradients the REFERENCE computes for them: torch autograd through
``avey_kernels.avey`` / ``avey_b`` with ``backend='torch'`` (the reference's
only differentiable path, ``avey_kernels/ops.py::_reference``) on CPU, for
every input that takes a gradient (z_tr, v, z_tl, bias). The reference
package is imported from ``--reference`` (or ``AVEY_REFERENCE``); it is needed
only to regenerate the fixtures.

Case families follow the reference's own gradient tests
(tests/test_contextualizer.py:41-62: fp64 gradcheck of Avey and Avey-B, NaN
padding that must not reach valid gradients) and widen them to every
activation, causal and bidirectional Avey, zero and sub-norm_eps rows, bias,
gate and padding masks, and fp32 / fp16 / bf16 inputs.

Usage: python tests/golden/make_grad_golden.py --reference <checkout of avey_kernel>
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from make_golden import encode  # noqa: E402

GRAD_FIELDS = ('z_tr', 'v', 'z_tl', 'bias')


def build_cases():
    cases = []

    def add(name, op, z_tr, *, v=None, z_tl=None, bias=None, valid=None, causal=True, eps=1e-6,
            activation='identity', seed=0):
        g = torch.Generator().manual_seed(seed)
        grad_out = torch.randn(z_tr.shape, generator=g).to(z_tr.dtype)
        cases.append(dict(name=name, op=op, z_tr=z_tr, v=v, z_tl=z_tl, bias=bias, valid=valid,
                          causal=causal, eps=eps, norm_eps=1e-12, activation=activation,
                          grad_out=grad_out))

    # fp64 (the reference's gradcheck dtype): NaN padding, a zero row and a row
    # whose norm is below norm_eps; every activation, both variants.
    g = torch.Generator().manual_seed(11)
    z = torch.randn(2, 9, 7, generator=g, dtype=torch.float64)
    z[0, 2] = 0
    z[1, 3] = 1e-13
    z[0, -1] = float('nan')
    zl = torch.randn(2, 9, 7, generator=g, dtype=torch.float64)
    zl[0, -1] = float('nan')
    bias = torch.randn(7, generator=g, dtype=torch.float64)
    v = torch.randn(9, 9, generator=g, dtype=torch.float64)
    valid = torch.ones(2, 9, dtype=torch.bool)
    valid[0, -1] = False
    valid[1, 5] = False
    for causal, act in ((True, 'identity'), (False, 'silu'), (True, 'relu')):
        add(f'f64_a_{act}_{int(causal)}', 'avey', z, v=v, z_tl=zl, bias=bias, valid=valid,
            causal=causal, activation=act, seed=1)
    for act in ('gelu', 'relu2', 'identity'):
        add(f'f64_b_{act}', 'avey_b', z, z_tl=zl, bias=bias, valid=valid, eps=0.25,
            activation=act, seed=2)
    # The reference's gradcheck inputs: no gate, bias or mask.
    g = torch.Generator().manual_seed(12)
    z = torch.rand(1, 3, 2, generator=g, dtype=torch.float64)
    add('f64_gradcheck_a', 'avey', z, v=torch.rand(3, 3, generator=g, dtype=torch.float64), seed=3)
    add('f64_gradcheck_b', 'avey_b', z, seed=3)
    # fp32, larger than one 32-wide tile, holes in the mask.
    g = torch.Generator().manual_seed(13)
    z = torch.randn(2, 45, 40, generator=g)
    valid = torch.rand(2, 45, generator=g) > 0.15
    add('f32_a_45', 'avey', z, v=torch.randn(45, 45, generator=g) * 0.1,
        z_tl=torch.randn(2, 45, 40, generator=g), bias=torch.randn(40, generator=g),
        valid=valid, activation='gelu', seed=4)
    add('f32_b_45', 'avey_b', z, z_tl=torch.randn(2, 45, 40, generator=g), valid=valid, eps=0.5,
        activation='silu', seed=5)
    # 16-bit inputs: the reference differentiates in fp32 and rounds the gradients.
    g = torch.Generator().manual_seed(14)
    for dt in (torch.bfloat16, torch.float16):
        x = torch.randn(2, 40, 64, generator=g)
        name = str(dt).replace('torch.', '')
        add(f'{name}_a', 'avey', x[..., 32:].to(dt), v=(torch.randn(40, 40, generator=g) * 0.05).to(dt),
            z_tl=x[..., :32].to(dt), bias=(torch.randn(32, generator=g) * 0.1).to(dt), seed=6)
        lengths = torch.tensor([40, 23])
        add(f'{name}_b', 'avey_b', x[..., 32:].to(dt), z_tl=x[..., :32].to(dt),
            valid=torch.arange(40)[None, :] < lengths[:, None], eps=0.5, activation='relu2', seed=7)
    return cases


def run_reference(case, ref):
    leaves = {k: (None if case[k] is None else case[k].clone().requires_grad_(True))
              for k in GRAD_FIELDS}
    kwargs = dict(z_tl=leaves['z_tl'], bias=leaves['bias'], valid=case['valid'],
                  norm_eps=case['norm_eps'], activation=case['activation'], backend='torch')
    if case['op'] == 'avey':
        out = ref.avey(leaves['z_tr'], leaves['v'], causal=case['causal'], **kwargs)
    else:
        out = ref.avey_b(leaves['z_tr'], eps=case['eps'], **kwargs)
    out.backward(case['grad_out'])
    return {k: (None if t is None else t.grad) for k, t in leaves.items()}


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument('--reference', default=os.environ.get('AVEY_REFERENCE'),
                        help='checkout of HusamettinYilmazz/avey_kernel (read-only is fine)')
    args = parser.parse_args()
    if not args.reference:
        parser.error('pass --reference or set AVEY_REFERENCE')
    sys.path.insert(0, args.reference)
    import avey_kernels as ref  # noqa: E402  (the reference package)

    torch.set_num_threads(1)
    arrays, manifest = {}, []
    for case in build_cases():
        grads = run_reference(case, ref)
        name = case['name']
        meta = dict(name=name, op=case['op'], dtype=str(case['z_tr'].dtype).replace('torch.', ''),
                    shape=list(case['z_tr'].shape), causal=case['causal'], eps=case['eps'],
                    norm_eps=case['norm_eps'], activation=case['activation'])
        for field in ('z_tr', 'v', 'z_tl', 'bias', 'valid', 'grad_out'):
            t = case[field]
            meta[field] = None if t is None else f'{name}/{field}'
            if t is not None:
                arrays[f'{name}/{field}'] = encode(t)
        for field, t in grads.items():
            meta['d_' + field] = None if t is None else f'{name}/d_{field}'
            if t is not None:
                arrays[f'{name}/d_{field}'] = encode(t)
        manifest.append(meta)
    np.savez_compressed(HERE / 'grad_golden.npz', **arrays)
    (HERE / 'grad_cases.json').write_text(json.dumps(manifest, indent=1) + '\n')
    print(f'wrote {len(manifest)} gradient cases')


if __name__ == '__main__':
    main()
