"""Generate the golden vectors in ``tests/golden/golden.npz`` + ``cases.json``.

Each case holds seeded inputs and the output of the REFERENCE implementation
itself: ``avey_kernels.avey`` / ``avey_kernels.avey_b`` with
``backend='torch'`` (which runs ``avey_kernels/ops.py::_reference``) on CPU.
The reference package is imported from a checkout given by ``--reference``
(default: the ``AVEY_REFERENCE`` environment variable); it is only needed to
regenerate the fixtures, never to run the tests.

Case families follow the reference's own tests:

* ``tiled_*``     tests/test_triton.py:126-160  (tails, zero row, NaN padding,
                  every activation, eps 0.25 for signed Avey-B inputs)
* ``lowprec_*``   tests/test_triton.py:97-124  (fp16/bf16 inputs, fp32 math)
* ``tiles_*``     tests/test_triton.py:70-95  (35x133 tails, gate, bias, mask)
* ``skip_*``      tests/test_causal_skip.py:80-105 (causal, NaN rows, silu)
* ``cfg1``        BASELINE config 1 (B=2, N=256, head/tail 128, fp32, seed 0)
* ``mini_*``      scaled-down bf16 versions of BASELINE configs 2-4
* ``edge_*``      one-token rows, fully padded rows, one-past-a-tile lengths

Usage: python tests/golden/make_golden.py --reference <checkout of avey_kernel>
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
DTYPES = {'float32': torch.float32, 'float16': torch.float16, 'bfloat16': torch.bfloat16}


def _case(name, op, z_tr, *, v=None, z_tl=None, bias=None, valid=None, causal=True,
          eps=1e-6, norm_eps=1e-12, activation='identity'):
    return dict(name=name, op=op, z_tr=z_tr, v=v, z_tl=z_tl, bias=bias, valid=valid,
                causal=causal, eps=eps, norm_eps=norm_eps, activation=activation)


def build_cases():
    cases = []
    # tests/test_triton.py:126-160 -- fp32, randn, tails, NaN padding, all activations.
    torch.manual_seed(17)
    for c, d in ((1, 1), (5, 7), (35, 37), (67, 65)):
        z_tr = torch.randn(2, c, d)
        z_tr[:, 0] = 0.
        z_tl = torch.randn_like(z_tr)
        bias = torch.randn(d)
        valid = torch.ones(2, c, dtype=torch.bool)
        if c > 1:
            valid[0, -1] = False
            valid[1] = False
            z_tr[0, -1] = float('nan')
        v = torch.randn(c, c)
        for normalized, causal, act in ((False, True, 'identity'), (False, False, 'silu'),
                                        (True, False, 'relu'), (True, False, 'gelu'),
                                        (True, False, 'relu2')):
            name = f'tiled_{c}x{d}_{"b" if normalized else "a"}_{act}_{int(causal)}'
            if normalized:
                cases.append(_case(name, 'avey_b', z_tr, z_tl=z_tl, bias=bias, valid=valid,
                                   eps=0.25, activation=act))
            else:
                cases.append(_case(name, 'avey', z_tr, v=v, z_tl=z_tl, bias=bias, valid=valid,
                                   causal=causal, activation=act))
    # tests/test_triton.py:97-124 -- low-precision inputs, no gate/bias/mask.
    torch.manual_seed(9)
    for dt in ('float16', 'bfloat16'):
        z_tr = torch.rand(2, 35, 37, dtype=DTYPES[dt])
        v = torch.randn(35, 35, dtype=DTYPES[dt])
        cases.append(_case(f'lowprec_{dt}_a', 'avey', z_tr, v=v))
        cases.append(_case(f'lowprec_{dt}_b', 'avey_b', z_tr))
    # tests/test_triton.py:70-95 -- 35 x 133 tails with gate, bias and mask.
    torch.manual_seed(29)
    for dt in ('float32', 'float16', 'bfloat16'):
        z_tr = torch.rand(2, 35, 133, dtype=DTYPES[dt])
        v = torch.randn(35, 35, dtype=DTYPES[dt])
        z_tl = torch.rand_like(z_tr)
        bias = torch.rand(133, dtype=DTYPES[dt])
        valid = torch.ones(2, 35, dtype=torch.bool)
        valid[0, -1] = False
        valid[1] = False
        cases.append(_case(f'tiles_{dt}_a', 'avey', z_tr, v=v, z_tl=z_tl, bias=bias, valid=valid))
        cases.append(_case(f'tiles_{dt}_b', 'avey_b', z_tr, z_tl=z_tl, bias=bias, valid=valid))
    # tests/test_causal_skip.py:80-105 -- causal Avey, NaN rows, silu, gate and bias.
    torch.manual_seed(43)
    for c, d in ((1, 7), (35, 37), (67, 133), (161, 37)):
        x = torch.randn(2, c, d)
        valid = torch.ones(2, c, dtype=torch.bool)
        valid[1] = False
        if c > 1:
            valid[0, -1] = False
        x[~valid] = float('nan')
        v, gate, bias = torch.randn(c, c), torch.randn_like(x), torch.randn(d)
        cases.append(_case(f'skip_{c}x{d}', 'avey', x, v=v, z_tl=gate, bias=bias, valid=valid,
                           activation='silu'))
    # B=2, N=256, enriched 256 = head 128 | tail 128, fp32, seed 0.
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 256, 256, generator=g)
    w = torch.randn(256, 256, generator=g) * 0.02
    cases.append(_case('cfg1', 'avey', x[..., 128:].contiguous(), v=w,
                       z_tl=x[..., :128].contiguous(), bias=torch.zeros(128)))
    # Scaled-down bf16 versions of configs 2-4 (same distributions, smaller shapes).
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 256, 384, generator=g)
    w = torch.randn(256, 256, generator=g) * 0.02
    bias = torch.randn(192, generator=g) * 0.01
    bf = torch.bfloat16
    cases.append(_case('mini_c2', 'avey', x[..., 192:].to(bf).contiguous(), v=w.to(bf),
                       z_tl=x[..., :192].to(bf).contiguous(), bias=bias.to(bf)))
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 256, 128, generator=g)
    lengths = torch.randint(64, 257, (3,), generator=g)
    valid = torch.arange(256)[None, :] < lengths[:, None]
    cases.append(_case('mini_c3', 'avey_b', x[..., 64:].to(bf).contiguous(),
                       z_tl=x[..., :64].to(bf).contiguous(), valid=valid))
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1, 384, 256, generator=g)
    w = torch.randn(384, 384, generator=g) * 0.02
    boost = torch.rand(1, 384, 1, generator=g) < 0.05
    x = torch.where(boost, x * 50, x)
    cases.append(_case('mini_c4', 'avey', x[..., 128:].to(bf).contiguous(), v=w.to(bf),
                       z_tl=x[..., :128].to(bf).contiguous()))
    # Edge cases: one token, one feature; an entirely padded batch row; 129 tokens
    # (one past a 128 tile) with a non-prefix mask and bf16 relu2.
    torch.manual_seed(5)
    cases.append(_case('edge_1x1', 'avey', torch.randn(1, 1, 1), v=torch.randn(1, 1)))
    z = torch.randn(2, 40, 16)
    valid = torch.ones(2, 40, dtype=torch.bool)
    valid[1] = False
    z[1] = float('nan')
    cases.append(_case('edge_allpad', 'avey_b', z, valid=valid, z_tl=torch.randn(2, 40, 16),
                       bias=torch.randn(16), eps=0.25))
    z = torch.rand(2, 129, 64, dtype=torch.bfloat16)
    valid = torch.rand(2, 129) > 0.2
    cases.append(_case('edge_129_holes', 'avey', z, v=torch.randn(129, 129, dtype=torch.bfloat16),
                       valid=valid, z_tl=torch.rand_like(z), activation='relu2'))
    cases.append(_case('edge_129_holes_b', 'avey_b', z, valid=valid, activation='gelu'))
    # Contexts above 512 (the long-context tensor-core path): more than one
    # group of 512 keys, a partial last tile, prefix padding past 512.
    g = torch.Generator().manual_seed(6)
    x = torch.randn(2, 640, 96, generator=g)
    lengths = torch.tensor([640, 530])
    valid = torch.arange(640)[None, :] < lengths[:, None]
    cases.append(_case('long_b_640', 'avey_b', x[..., 48:].to(bf).contiguous(),
                       z_tl=x[..., :48].to(bf).contiguous(), valid=valid, activation='gelu'))
    x = torch.randn(1, 520, 64, generator=g)
    w = torch.randn(520, 520, generator=g) * 0.05
    bias = torch.randn(32, generator=g) * 0.1
    cases.append(_case('long_a_520', 'avey', x[..., 32:].to(bf).contiguous(), v=w.to(bf),
                       z_tl=x[..., :32].to(bf).contiguous(), bias=bias.to(bf)))
    return cases


def encode(t: torch.Tensor) -> np.ndarray:
    """Store bf16 as its raw 16-bit pattern (uint16); other dtypes natively."""
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def run_reference(case, ref):
    kwargs = dict(z_tl=case['z_tl'], bias=case['bias'], valid=case['valid'],
                  norm_eps=case['norm_eps'], activation=case['activation'], backend='torch')
    if case['op'] == 'avey':
        return ref.avey(case['z_tr'], case['v'], causal=case['causal'], **kwargs)
    return ref.avey_b(case['z_tr'], eps=case['eps'], **kwargs)


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
    arrays, manifest, stored = {}, [], {}
    for case in build_cases():
        with torch.no_grad():
            out = run_reference(case, ref)
        name = case['name']
        meta = dict(name=name, op=case['op'], dtype=str(case['z_tr'].dtype).replace('torch.', ''),
                    shape=list(case['z_tr'].shape), causal=case['causal'], eps=case['eps'],
                    norm_eps=case['norm_eps'], activation=case['activation'])
        for field in ('z_tr', 'v', 'z_tl', 'bias', 'valid'):
            t = case[field]
            if t is None:
                meta[field] = None
                continue
            # Cases of one family share input tensors: store each tensor once.
            if id(t) not in stored:
                key = f'in{len(stored)}'
                stored[id(t)] = key
                arrays[key] = encode(t)
            meta[field] = stored[id(t)]
        arrays[f'{name}/out'] = encode(out)
        manifest.append(meta)
    np.savez_compressed(HERE / 'golden.npz', **arrays)
    (HERE / 'cases.json').write_text(json.dumps(manifest, indent=1) + '\n')
    print(f'wrote {len(manifest)} cases to {HERE}')


if __name__ == '__main__':
    main()
