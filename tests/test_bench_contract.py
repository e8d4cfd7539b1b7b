"""bench.py's host-side contract, checked on CPU.

The GPU arm needs a B200; the reference arm (the CPU implementation of the
path, timed on the host) and the pure helpers run here: the JSON line's keys,
the algorithmic byte and FLOP counts quoted in the roofline, and the batch
split of the strong-scaling config.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_reference_arm_prints_one_json_line_with_the_contract_keys():
    env = dict(os.environ, WORLD_SIZE='1', RANK='0', LOCAL_RANK='0')
    res = subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference',
                          '--steps', '1', '--warmup', '0'],
                         capture_output=True, text=True, env=env, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ('impl', 'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step',
                'higher_is_better', 'config', 'cpu_baseline', 'e2e'):
        assert key in line, key
    assert line['impl'] == 'reference' and line['value'] > 0 and line['higher_is_better']
    assert line['e2e']['h2d_bytes_per_step'] == 0 and line['e2e']['value'] == line['value']
    # The reference's own CPU path when its unmodified install is importable,
    # else the NumPy port of it.
    ref_installed = (ROOT / 'baseline' / '_ref' / 'avey_kernels' / 'ops.py').exists()
    assert line['cpu_baseline']['kind'] == ('reference' if ref_installed else 'port')
    assert line['cpu_baseline']['cores'] >= 1
    assert line['config']['workload'].startswith('c2:')
    assert line['config']['global_batch'] == 64


def test_algorithmic_bytes_and_flops_of_config_2():
    cfg = bench.CONFIGS['c2']
    nbytes, flops = bench.algorithmic(cfg, 64, None)
    assert nbytes == 2 * 64 * 512 * 768 * 3 + 2 * 512 * 512 + 2 * 768 == 151_520_768
    assert flops == 4 * 768 * 64 * (512 * 513 // 2)


def test_algorithmic_counts_with_a_padding_mask():
    cfg = dict(bench.CONFIGS['c3'])
    valid = torch.zeros(2, 512, dtype=torch.bool)
    valid[0, :100] = True
    valid[1, :512] = True
    nbytes, flops = bench.algorithmic(cfg, 2, valid)
    assert flops == 4 * 384 * (100 * 100 + 512 * 512)
    assert nbytes == 2 * 2 * 512 * 384 * 3 + 2 * 512


@pytest.mark.parametrize('world', [1, 2, 4, 8])
def test_strong_scaling_config_splits_the_global_batch(world):
    assert bench.shard_batch(bench.CONFIGS['c5'], world) == 1024 // world
    assert bench.shard_batch(bench.CONFIGS['c2'], world) == 64  # weak scaling: fixed per GPU
