"""Host logic of the many-network path: how networks are sharded over ranks (no GPU).

The multi-GPU form of the batched networks is replicas with no collective:
each rank trains ``shard(nets, world, rank)``.  Checked: the shards of every
rank cover each network exactly once, are contiguous and balanced, and two
gloo ranks agree on the split.
"""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from lich_b200.many_nets import shard


@pytest.mark.parametrize("nets", [1, 7, 4096, 4097])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_cover_every_network_once(nets, world):
    parts = [shard(nets, world, r) for r in range(world)]
    flat = [n for p in parts for n in p]
    assert flat == list(range(nets))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_bad_requests():
    for args in ((-1, 2, 0), (4, 0, 0), (4, 2, 2)):
        with pytest.raises(ValueError):
            shard(*args)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard(4096, world, rank)
        got = [None] * world
        dist.all_gather_object(got, (mine.start, mine.stop))
        out[rank] = got
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_agree_on_the_split():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.get_context("spawn").Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
        res = dict(out)
    assert res[0] == res[1] == [(0, 2048), (2048, 4096)]
