"""Host logic of the multi-GPU path, on CPU: the batch*head partition, and a world-size-2
gloo run that computes each rank's slice independently (no collective on the data path) and
gathers the slices afterwards only to check them."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from mini_flash_attention.sharding import all_shards, bh_shard


@pytest.mark.parametrize("total,world", [(8, 1), (8, 2), (8, 8), (256, 8), (7, 3), (3, 4),
                                         (2048, 8), (32, 8)])
def test_shards_cover_rows_once_contiguously(total, world):
    shards = all_shards(total, world)
    assert shards[0].start == 0 and shards[-1].stop == total
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    sizes = [s.rows for s in shards]
    assert max(sizes) - min(sizes) <= 1
    assert sum(sizes) == total


def test_bad_rank_rejected():
    with pytest.raises(ValueError):
        bh_shard(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist

    from make_golden import make_inputs
    from oracle.attention import naive_attention

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v = (x.reshape(6, 128, 64) for x in make_inputs((2, 3, 128, 64), "normal", 3))
    sh = bh_shard(6, rank, world)
    local = naive_attention(q[sh.start:sh.stop], k[sh.start:sh.stop], v[sh.start:sh.stop])
    # validation only, outside any timed region: gather the slices on every rank
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([sh.rows]))
    pieces = [torch.zeros((int(s.item()), 128, 64)) for s in sizes]
    dist.all_gather(pieces, torch.from_numpy(np.ascontiguousarray(local)).float())
    if rank == 0:
        full = torch.cat(pieces).numpy()
        want = naive_attention(q, k, v)
        result_q.put(float(np.max(np.abs(full - want))))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_sharded_forward_matches_full():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 0.0
