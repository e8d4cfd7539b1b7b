import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / 'tests' / 'golden'
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (sm_100a) and the built CUDA library')


def pytest_collection_modifyitems(config, items):
    # A GPU test must fail loudly on a GPU box without the library, but is
    # skipped here (no CUDA device) when selected without -m "not gpu".
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason='no CUDA device in this process')
    for item in items:
        if 'gpu' in item.keywords:
            item.add_marker(skip)


def pytest_sessionstart(session):
    # Build the native library in-tree when it is missing or stale (nvcc
    # cross-compiles for sm_100a without a GPU). On the GPU box the prebuilt
    # library travels with the repository and is reused.
    from avey_kernel_b200.csrc import build
    try:
        build.build()
    except Exception as exc:  # surfaced by the tests that need the library
        session.config._avey_build_error = exc  # noqa: SLF001
