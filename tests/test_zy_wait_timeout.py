"""The failure path of the tensor-core kernels: a bounded wait that runs out.

Every mbarrier wait in the library's kernels gives up after a cycle limit,
raises AVEY_DEVFLAG_TIMEOUT and unwinds, so a kernel whose producer never
arrives still returns and frees its tensor memory instead of hanging. Here the
test hooks (avey_test_hooks_v1) lower the limit to 10^5 cycles and make the
fused kernel's TMA and MMA warps issue nothing, so no TMA is ever in flight and
its compute warps' wait for the Gram runs out. Nothing faults or traps: the
call returns, the status word reports the timeout, and after clearing it the
next normal call on the same context is correct.

Collected just before test_zz_no_alloc.py; the hooks are restored even when an
assertion fails.
"""

import numpy as np
import pytest
import torch

from avey_kernel_b200 import _native, ops
from helpers import TOL, norm_rel_err, to_numpy

import oracle

TIMEOUT = 1  # AVEY_DEVFLAG_TIMEOUT


@pytest.mark.gpu
def test_a_wait_that_runs_out_raises_the_flag_and_the_context_stays_usable():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 256, 2 * 128, generator=g).to(torch.bfloat16).cuda()
    head, tail = x[..., :128], x[..., 128:]
    plan = ops.plan(tail, None, head, causal=False, normalize=True)
    assert plan.kernel == _native.KERNEL_TCGEN05 and plan.launches == 1  # the fused kernel
    assert _native.device_status(clear=True) == 0
    try:
        _native.test_hooks(100_000, stall=True)
        ops.avey_b(tail, z_tl=head, backend='cuda')  # returns; its output is not defined
        torch.cuda.synchronize()
        assert _native.device_status(clear=True) & TIMEOUT
    finally:
        _native.test_hooks()
        _native.device_status(clear=True)
    out = ops.avey_b(tail, z_tl=head, backend='cuda')
    torch.cuda.synchronize()
    want = oracle.avey_b(to_numpy(tail), z_tl=to_numpy(head))
    assert np.isfinite(to_numpy(out)).all()
    assert norm_rel_err(to_numpy(out), want) <= TOL['bfloat16']
    assert _native.device_status() == 0
