"""The multi-GPU host path on the CPU: gloo process groups, world size 2.

A run on N GPUs gives each rank a contiguous batch shard and has no
collective on the data path (planes are independent,
kernels/vectra_kernels/spatial_rbf_attention.py:237); these tests check the
host logic around it with the float64 oracle standing in for the kernel:
shards partition the batch, broadcast arguments are shared, gathering the
shards in rank order reproduces the whole-batch result bit for bit, the
timing reduction takes the slowest rank, and a rank that fails is reported
instead of leaving the others waiting.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vectra_b200 import sharding


@pytest.mark.parametrize('n', [0, 1, 7, 8, 1023, 1024])
@pytest.mark.parametrize('world', [1, 2, 3, 8])
def test_shard_ranges_partition_the_batch(n, world):
    rows = []
    for r in range(world):
        lo, hi = sharding.shard_range(n, world, r)
        assert 0 <= hi - lo <= -(-n // world)
        rows.extend(range(lo, hi))
    assert rows == list(range(n))


def test_shard_range_rejects_bad_ranks():
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)
    with pytest.raises(ValueError):
        sharding.shard_range(-1, 2, 0)


def test_shard_args_slices_batch_and_shares_broadcasts():
    q = torch.zeros(5, 2, 1, 4)
    k = v = torch.zeros(5, 2, 3, 4)
    per_head = torch.ones(1, 2, 1, 1)
    per_row_bias = torch.arange(5.).view(5, 1, 1, 1).expand(5, 1, 1, 3)
    a = sharding.shard_args(q, k, v, per_head, per_row_bias, 2, 1)
    assert a[0].shape[0] == 2 and a[1].shape[0] == 2
    assert a[3] is per_head
    assert a[4][:, 0, 0, 0].tolist() == [3.0, 4.0]
    scalar = torch.tensor(0.5)
    assert sharding.shard_args(q, k, v, scalar, None, 2, 0)[3] is scalar


def test_single_process_collectives_are_identities():
    t = torch.arange(6.).view(3, 2)
    assert sharding.max_over_ranks(2.5) == 2.5
    assert sharding.gather_rows(t, 3) is t


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_total):
    # Children start with `spawn`: a fresh interpreter, no inherited state.
    from oracle import rbf_oracle  # pylint: disable=import-outside-toplevel
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(11)
        q = torch.randn(n_total, 3, 1, 8, generator=gen)
        k = torch.randn(n_total, 3, 12, 8, generator=gen)
        v = torch.randn(n_total, 3, 12, 8, generator=gen)
        scale = 0.2 + torch.rand(1, 3, 1, 1, generator=gen)
        bias = torch.zeros(n_total, 1, 1, 12)
        for b in range(n_total):
            bias[b, ..., 2 + b % 10:] = float('-inf')
        sq, sk, sv, ss, sb = sharding.shard_args(q, k, v, scale, bias,
                                                 world, rank)
        mine = torch.from_numpy(rbf_oracle.expanded_rbf_attention(
            sq.numpy(), sk.numpy(), sv.numpy(), ss.numpy(), sb.numpy()))
        full = sharding.gather_rows(mine, n_total)
        whole = rbf_oracle.expanded_rbf_attention(
            q.numpy(), k.numpy(), v.numpy(), scale.numpy(), bias.numpy())
        assert full.shape == whole.shape
        assert np.array_equal(full.numpy(), whole), 'gathered shards differ'
        slowest = sharding.max_over_ranks(1.5 + rank)
        assert slowest == 1.5 + (world - 1), slowest
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('n_total', [7, 8])
def test_two_ranks_reproduce_the_whole_batch(n_total):
    mp.start_processes(_worker, args=(2, _free_port(), n_total), nprocs=2,
                       join=True, start_method='spawn')


def _dying_worker(rank, world, port):
    import datetime  # pylint: disable=import-outside-toplevel
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        if rank == 1:
            raise RuntimeError('rank 1 fails before the gather')
        sharding.gather_rows(torch.zeros(2, 3), 4)
    finally:
        dist.destroy_process_group()


def test_a_rank_that_dies_is_reported_not_waited_for():
    # A rank that fails between steps: the launcher reports an error (the
    # failed rank's own, or the surviving rank's broken collective, which
    # ever arrives first) well before the process group's 20 s timeout.
    import time  # pylint: disable=import-outside-toplevel
    t0 = time.monotonic()
    # Either report counts: an exception raised in a rank, or a rank that
    # exited abnormally.
    with pytest.raises((mp.ProcessRaisedException,
                        mp.ProcessExitedException)):
        mp.start_processes(_dying_worker, args=(2, _free_port()), nprocs=2,
                           join=True, start_method='spawn')
    assert time.monotonic() - t0 < 18


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    import bench  # pylint: disable=import-outside-toplevel
    monkeypatch.setenv('RANK', '1')
    assert bench.main(['--impl', 'reference', '--gpus', '2', '--steps', '1',
                       '--warmup', '0']) == 0
    assert capsys.readouterr().out == ''
