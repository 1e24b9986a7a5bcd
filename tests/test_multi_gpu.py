"""The operator on two or more GPUs (skipped with fewer): one process per
GPU over NCCL, each rank computing its contiguous batch shard of the same
seeded inputs; the gathered shards must equal the one-GPU result bit for
bit (planes are independent, so sharding changes no arithmetic). The
kernels are plain launches per rank: no collective on the data path.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, config, batch):
    import datetime  # pylint: disable=import-outside-toplevel
    import vectra_b200  # pylint: disable=import-outside-toplevel
    from vectra_b200 import sharding  # pylint: disable=import-outside-toplevel
    from vectra_b200 import workloads  # pylint: disable=import-outside-toplevel
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    os.environ['NCCL_NVLS_ENABLE'] = '0'
    torch.cuda.set_device(rank)
    dev = torch.device('cuda', rank)
    dist.init_process_group('nccl', rank=rank, world_size=world,
                            device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        w = workloads.make(config, device=dev, seed=5, batch=batch)
        args = sharding.shard_args(*w.tensors(), world, rank)
        mine = vectra_b200.rbf_attention(*args)
        full = sharding.gather_rows(mine, batch)
        if rank == 0:
            whole = vectra_b200.rbf_attention(*w.tensors())
            assert torch.equal(full.isnan(), whole.isnan())
            assert torch.equal(full.nan_to_num(), whole.nan_to_num())
        slowest = sharding.max_over_ranks(float(rank), device=dev)
        assert slowest == float(world - 1)
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs 2 GPUs')
@pytest.mark.parametrize('config,batch', [(2, 1024), (2, 37), (3, 301)])
def test_shards_reproduce_the_single_gpu_result(config, batch):
    world = min(torch.cuda.device_count(), 8)
    mp.start_processes(_worker, args=(world, _free_port(), config, batch),
                       nprocs=world, join=True, start_method='spawn')
