"""Build ``avey_kernel_b200/lib/libavey_b200.so`` with nvcc for sm_100a.

Usage: python -m avey_kernel_b200.csrc.build [--force] [--verbose]
The library exports only the C ABI declared in ``include/avey_b200.h``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
LIB_DIR = PKG / 'lib'
LIB = LIB_DIR / 'libavey_b200.so'
SOURCES = ['avey_api.cu', 'avey_bwd.cu']
HEADERS = ['ptx.cuh', 'common.cuh', 'norm_prepass.cuh', 'simt_kernel.cuh', 'simt2_kernel.cuh',
           'small_kernel.cuh', 'tc_kernel.cuh', 'tc_long.cuh', 'tc_tf32.cuh', 'tc_gemm.cuh', 'bwd_kernels.cuh']

NVCC_FLAGS = [
    '-gencode', 'arch=compute_100a,code=sm_100a',
    '-O3', '-lineinfo', '-std=c++17',
    '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
    '--expt-relaxed-constexpr',
    '-shared',
]


def nvcc_path() -> str:
    home = os.environ.get('CUDA_HOME', '/usr/local/cuda')
    cand = Path(home) / 'bin' / 'nvcc'
    if cand.exists():
        return str(cand)
    found = shutil.which('nvcc')
    if not found:
        raise RuntimeError('nvcc not found (set CUDA_HOME)')
    return found


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / 'include' / 'avey_b200.h']
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False, extra=()) -> Path:
    """Build the library unless it is newer than every source."""
    target = LIB
    if not force and not needs_build():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = target.with_suffix('.so.tmp')
    cmd = [nvcc_path(), *NVCC_FLAGS, *extra, '-I', str(ROOT / 'include'), '-I', str(CSRC),
           *[str(CSRC / s) for s in SOURCES], '-o', str(tmp), '-lcudart']
    if verbose:
        print(' '.join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f'nvcc failed with exit code {res.returncode}')
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    os.replace(tmp, target)
    return target


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas-info', action='store_true', help='print registers / spills / smem')
    args = ap.parse_args()
    extra = ['-Xptxas', '-v'] if args.ptxas_info else []
    print(build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info,
                extra=extra))


if __name__ == '__main__':
    main()
