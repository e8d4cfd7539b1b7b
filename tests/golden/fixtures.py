"""Loader for the golden vectors written by ``make_golden.py``.

``load_cases()`` returns dicts with float32/bool NumPy inputs (bf16 and fp16
values are exact in float32), the case's dtype name, its flags, and the
reference output (rounded to the case dtype by the reference, widened here).
``to_torch(case, device)`` rebuilds the inputs as tensors of the case dtype.
"""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
FIELDS = ('z_tr', 'v', 'z_tl', 'bias', 'valid')


def _decode(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.uint16:  # raw bfloat16 bits
        return (a.astype(np.uint32) << 16).view(np.float32)
    if a.dtype == np.float16:
        return a.astype(np.float32)
    return a


@lru_cache(maxsize=1)
def load_cases():
    manifest = json.loads((HERE / 'cases.json').read_text())
    data = np.load(HERE / 'golden.npz')
    cases = []
    for meta in manifest:
        case = dict(meta)
        for field in FIELDS:
            key = meta[field]
            case[field] = None if key is None else _decode(data[key])
        case['out'] = _decode(data[meta['name'] + '/out'])
        cases.append(case)
    return tuple(cases)


def case_by_name(name: str) -> dict:
    for case in load_cases():
        if case['name'] == name:
            return case
    raise KeyError(name)


def to_torch(case: dict, device='cpu'):
    """Inputs as torch tensors of the case dtype on ``device``."""
    import torch
    dtype = getattr(torch, case['dtype'])
    out = {}
    for field in FIELDS:
        a = case[field]
        if a is None:
            out[field] = None
        elif a.dtype == np.bool_:
            out[field] = torch.from_numpy(a.copy()).to(device)
        else:
            out[field] = torch.from_numpy(a.copy()).to(device=device, dtype=dtype)
    return out


def oracle_kwargs(case: dict) -> dict:
    """Keyword arguments for ``oracle.contextualize`` from a case's flags."""
    return dict(eps=case['eps'] if case['op'] == 'avey_b' else 1e-6,
                norm_eps=case['norm_eps'],
                causal=case['causal'] if case['op'] == 'avey' else False,
                normalize=case['op'] == 'avey_b', activation=case['activation'])


GRAD_FIELDS = ('z_tr', 'v', 'z_tl', 'bias')


@lru_cache(maxsize=1)
def load_grad_cases():
    """Gradient cases of ``make_grad_golden.py``: inputs, ``grad_out`` and the
    reference's gradients ``d_<input>`` (None where the input is absent)."""
    manifest = json.loads((HERE / 'grad_cases.json').read_text())
    data = np.load(HERE / 'grad_golden.npz')
    cases = []
    for meta in manifest:
        case = dict(meta)
        for field in FIELDS + ('grad_out',) + tuple('d_' + f for f in GRAD_FIELDS):
            key = meta[field]
            case[field] = None if key is None else _decode(data[key])
        cases.append(case)
    return tuple(cases)


def grad_to_torch(case: dict, device='cpu'):
    """Inputs and grad_out as tensors of the case dtype on ``device``."""
    out = to_torch(case, device)
    import torch
    out['grad_out'] = torch.from_numpy(case['grad_out'].copy()).to(
        device=device, dtype=getattr(torch, case['dtype']))
    return out
