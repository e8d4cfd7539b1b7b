"""Multi-rank host logic (batch shards, max over ranks, gather to rank 0).

The data path has no collective: each rank runs the single-GPU forward on its
contiguous batch shard. These tests run two gloo ranks on CPU (the forward
takes the PyTorch path there) and check that the shards, put back together
on rank 0, are the full-batch result, and that the timing reduction is a max.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from avey_kernel_b200 import shard


def test_shard_bounds_cover_the_batch_in_order():
    for world in (1, 2, 4, 8):
        bounds = [shard.shard_bounds(64, world, r) for r in range(world)]
        assert bounds[0][0] == 0 and bounds[-1][1] == 64
        assert all(a[1] == b[0] for a, b in zip(bounds, bounds[1:]))
        assert len({stop - start for start, stop in bounds}) == 1


@pytest.mark.parametrize('args', [(10, 4, 0), (8, 0, 0), (8, 2, 2), (8, 2, -1)])
def test_shard_bounds_reject_bad_splits(args):
    with pytest.raises(ValueError):
        shard.shard_bounds(*args)


def test_single_process_reductions_are_identities():
    t = torch.arange(6.0)
    assert shard.max_over_ranks(3.5) == 3.5
    assert shard.gather_to_rank0(t)[0] is t
    assert shard.shard(t.view(3, 2), 1, 0).data_ptr() == t.data_ptr()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from avey_kernel_b200 import avey, avey_b
        assert shard.rank_env() == (world, rank, rank)
        g = torch.Generator().manual_seed(5)
        b, n, d = 4, 24, 16
        x = torch.randn(b, n, 2 * d, generator=g, dtype=torch.float64)
        v = torch.randn(n, n, generator=g, dtype=torch.float64)
        lengths = torch.tensor([24, 7, 16, 1])
        valid = torch.arange(n)[None, :] < lengths[:, None]
        mine, my_valid = shard.shard(x, world, rank), shard.shard(valid, world, rank)
        y_avey = avey(mine[..., d:], v, z_tl=mine[..., :d], backend='torch')
        y_b = avey_b(mine[..., d:], z_tl=mine[..., :d], valid=my_valid, backend='torch')
        parts_avey = shard.gather_to_rank0(y_avey)
        parts_b = shard.gather_to_rank0(y_b)
        slowest = shard.max_over_ranks(0.25 * (rank + 1))
        result = dict(slowest=slowest, got_parts=parts_avey is not None)
        if rank == 0:
            result.update(
                avey=torch.cat(parts_avey), avey_full=avey(x[..., d:], v, z_tl=x[..., :d],
                                                           backend='torch'),
                avey_b=torch.cat(parts_b),
                avey_b_full=avey_b(x[..., d:], z_tl=x[..., :d], valid=valid, backend='torch'))
        torch.save(result, os.path.join(outdir, f'rank{rank}.pt'))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_full_batch(tmp_path):
    world = 2
    ctx = mp.get_context('spawn')
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0] * world
    r0 = torch.load(tmp_path / 'rank0.pt')
    r1 = torch.load(tmp_path / 'rank1.pt')
    assert r0['slowest'] == r1['slowest'] == 0.5
    assert r0['got_parts'] and not r1['got_parts']
    torch.testing.assert_close(r0['avey'], r0['avey_full'], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(r0['avey_b'], r0['avey_b_full'], rtol=1e-12, atol=1e-12)
