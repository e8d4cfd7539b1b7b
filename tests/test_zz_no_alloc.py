"""avey_fwd_noalloc_v1: the entry point for callers that cannot allocate.

Some callers hold no device allocator of their own (an FFI host that only
hands raw pointers over, or code running while a stream is captured into a
CUDA graph, where allocation is not allowed). For them the library keeps its
scratch -- one float per row of z_tr -- in an array of its own, up to
AVEY_NOALLOC_MAX_ROWS rows. These tests call that entry point through the C
ABI and check it against avey_fwd_v1 on calls in a row: a later call finds an
earlier call's sums still in the shared array and must not depend on them.
On the fused tensor-core path this entry point runs the kernel's pre-pass
variant (row sums in the array) where avey_fwd_v1 sums the rows inside the
kernel, so the two agree within the bf16 tolerance, and a repeated call of
this entry point agrees with itself bit for bit.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""

import numpy as np
import pytest
import torch

from avey_kernel_b200 import _native, ops
from helpers import TOL, norm_rel_err, to_numpy


def _call(z_tr, v, z_tl, bias, valid, *, causal, normalize, act, noalloc, kernel=0):
    out = torch.empty(z_tr.shape, dtype=z_tr.dtype, device=z_tr.device)
    params = ops.build_params(z_tr, v, z_tl, bias, valid, out, eps=1e-6, norm_eps=1e-12,
                              causal=causal, normalize=normalize, activation_id=act, kernel=kernel)
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        _native.forward_noalloc(params, stream)  # params.workspace stays NULL
    else:
        nbytes = _native.workspace_size(params)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=z_tr.device)
        params.workspace = ws.data_ptr()
        params.workspace_bytes = nbytes
        _native.forward(params, stream)
    torch.cuda.synchronize()
    return out


@pytest.mark.gpu
def test_noalloc_entry_point_matches_the_workspace_entry_point_on_two_calls():
    g = torch.Generator().manual_seed(11)
    cases = [
        # Avey causal, bf16, BASELINE-config-2-like (tcgen05 path, uses scratch)
        dict(b=8, n=512, d=768, causal=True, normalize=False, act=0, weight=True, mask=False),
        # Avey-B, bf16, ragged padding, gelu -- fewer rows than the first call,
        # so the array still holds the first call's sums past these rows
        dict(b=3, n=384, d=256, causal=False, normalize=True, act=4, weight=False, mask=True),
    ]
    first = None
    for c in cases:
        x = torch.randn(c['b'], c['n'], 2 * c['d'], generator=g).to(torch.bfloat16).cuda()
        head, tail = x[..., :c['d']], x[..., c['d']:]
        v = ((torch.randn(c['n'], c['n'], generator=g) * 0.02).to(torch.bfloat16).cuda()
             if c['weight'] else None)
        valid = None
        if c['mask']:
            lengths = torch.randint(c['n'] // 4, c['n'] + 1, (c['b'],), generator=g)
            valid = (torch.arange(c['n'])[None, :] < lengths[:, None]).cuda()
        plan = ops.plan(tail, v, head, None, valid, causal=c['causal'], normalize=c['normalize'])
        assert plan.kernel == _native.KERNEL_TCGEN05
        kw = dict(causal=c['causal'], normalize=c['normalize'], act=c['act'])
        want = _call(tail, v, head, None, valid, noalloc=False, **kw)
        got = _call(tail, v, head, None, valid, noalloc=True, **kw)
        assert np.isfinite(to_numpy(got)).all()
        assert norm_rel_err(to_numpy(got), to_numpy(want)) <= TOL['bfloat16']
        if first is None:
            first = (tail, v, head, valid, kw, got)
    # The first case again, after the second left its sums in the array: the
    # same bits as its first call.
    tail, v, head, valid, kw, got = first
    assert torch.equal(_call(tail, v, head, None, valid, noalloc=True, **kw), got)
    assert _native.device_status(clear=True) == 0


@pytest.mark.gpu
def test_noalloc_entry_point_on_the_cuda_core_path():
    z = torch.rand(2, 35, 37, device='cuda')
    want = _call(z, None, None, None, None, causal=False, normalize=True, act=0, noalloc=False)
    got = _call(z, None, None, None, None, causal=False, normalize=True, act=0, noalloc=True)
    assert norm_rel_err(to_numpy(got), to_numpy(want)) <= TOL['float32']


@pytest.mark.gpu
def test_noalloc_entry_point_runs_fp32_on_cuda_cores():
    # avey_fwd_v1 runs aligned fp32 on the 3xTF32 kernel pair, whose P
    # workspace the no-allocation entry point does not have: it takes the
    # CUDA-core kernel, within the fp32 bound of the pair's result.
    z = torch.rand(2, 96, 72, device='cuda')
    assert ops.plan(z, causal=False, normalize=True).kernel == _native.KERNEL_TCGEN05
    want = _call(z, None, z, None, None, causal=False, normalize=True, act=0, noalloc=False)
    got = _call(z, None, z, None, None, causal=False, normalize=True, act=0, noalloc=True)
    assert norm_rel_err(to_numpy(got), to_numpy(want)) <= TOL['float32']


def test_noalloc_entry_point_rejects_inputs_beyond_its_limit():
    # 2049 x 512 rows on the fused tensor-core path (the one that reads the
    # scratch) is past the limit; rejected before anything launches.
    z = torch.empty(_native.NOALLOC_MAX_ROWS // 512 + 1, 512, 8, dtype=torch.bfloat16)
    out = torch.empty_like(z)
    params = ops.build_params(z, None, None, None, None, out, eps=1e-6, norm_eps=1e-12,
                              causal=False, normalize=True, activation_id=0)
    before = _native.launch_count()
    with pytest.raises(_native.NativeError, match='no-allocation limit'):
        _native.forward_noalloc(params, 0)
    assert _native.launch_count() == before


@pytest.mark.gpu
def test_noalloc_entry_point_runs_small_fp32_on_the_8_row_kernel():
    # Small fp32 problems run the 8-row CUDA-core kernel on both entry points
    # (it needs no workspace): the results agree bit for bit.
    z = torch.rand(2, 96, 64, device='cuda')
    plan = ops.plan(z, causal=False, normalize=True)
    assert plan.kernel == _native.KERNEL_SIMT and plan.reason == _native.REASON_SMALL
    before = _native.launch_count()
    got = _call(z, None, z, None, None, causal=False, normalize=True, act=0, noalloc=True)
    assert _native.launch_count() == before + 1
    want = _call(z, None, z, None, None, causal=False, normalize=True, act=0, noalloc=False)
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_noalloc_entry_point_runs_long_contexts_on_cuda_cores():
    # Above 512 tokens avey_fwd_v1 takes the long-context tcgen05 path, whose
    # P workspace this entry point does not have: it runs the CUDA-core kernel.
    z = torch.randn(1, 600, 64, device='cuda').to(torch.bfloat16)
    plan = ops.plan(z, causal=False, normalize=True)
    assert plan.kernel == _native.KERNEL_TCGEN05 and plan.launches == 3
    before = _native.launch_count()
    got = _call(z, None, None, None, None, causal=False, normalize=True, act=0, noalloc=True)
    assert _native.launch_count() == before + 1
    want = _call(z, None, None, None, None, causal=False, normalize=True, act=0, noalloc=False)
    assert norm_rel_err(to_numpy(got), to_numpy(want)) <= TOL['bfloat16']


@pytest.mark.gpu
def test_noalloc_entry_point_runs_cuda_core_inputs_past_the_row_limit():
    # The CUDA-core kernels read no scratch, so the row limit does not apply:
    # fp32 input with more rows than the array holds. avey_fwd_v1 would run
    # fp32 on the 3xTF32 tensor-core pair (with a P workspace); this entry
    # point runs it on CUDA cores, so the bitwise comparison forces that
    # kernel on the workspace entry point too.
    z = torch.rand(_native.NOALLOC_MAX_ROWS // 64 + 1, 64, 8, device='cuda')
    got = _call(z, None, None, None, None, causal=False, normalize=True, act=0, noalloc=True)
    want = _call(z, None, None, None, None, causal=False, normalize=True, act=0, noalloc=False,
                 kernel=_native.KERNEL_SIMT)
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_noalloc_entry_point_replays_from_a_cuda_graph():
    # Graph capture is one of the situations with no allocator: warm up once
    # (the first call on a device looks up the scratch address), capture one
    # call into a CUDA graph, replay it, and compare with an eager call of the
    # same entry point bit for bit, and with avey_fwd_v1 within the tolerance.
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 512, 2 * 256, generator=g).to(torch.bfloat16).cuda()
    head, tail = x[..., :256], x[..., 256:]
    v = (torch.randn(512, 512, generator=g) * 0.02).to(torch.bfloat16).cuda()
    plain = _call(tail, v, head, None, None, causal=True, normalize=False, act=3, noalloc=False)
    want = _call(tail, v, head, None, None, causal=True, normalize=False, act=3, noalloc=True)
    assert norm_rel_err(to_numpy(want), to_numpy(plain)) <= TOL['bfloat16']
    out = torch.full(tail.shape, float('nan'), dtype=tail.dtype, device='cuda')
    params = ops.build_params(tail, v, head, None, None, out, eps=1e-6, norm_eps=1e-12,
                              causal=True, normalize=False, activation_id=3)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            _native.forward_noalloc(params, side.cuda_stream)
    torch.cuda.current_stream().wait_stream(side)
    out.fill_(float('nan'))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    out.fill_(float('nan'))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    del graph
