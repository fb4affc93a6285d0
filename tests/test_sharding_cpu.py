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


# ---- query-row sharding (fewer batch*head rows than ranks)
from mini_flash_attention.sharding import Q_ALIGN, q_shard, shard_mode  # noqa: E402


@pytest.mark.parametrize("n,world", [(65536, 2), (65536, 8), (8192, 3), (1000, 8), (1, 4),
                                     (257, 2), (0, 2), (4096, 16)])
def test_query_shards_cover_rows_once_in_whole_units(n, world):
    shards = [q_shard(n, r, world) for r in range(world)]
    assert shards[0].begin == 0 and shards[-1].end == n
    for a, b in zip(shards, shards[1:]):
        assert a.end == b.begin
    for s in shards:
        assert 0 <= s.begin <= s.end <= n
        assert s.begin % Q_ALIGN == 0 or s.begin == n
    blocks = [-(-s.rows // Q_ALIGN) for s in shards]
    assert max(blocks) - min(blocks) <= 1


@pytest.mark.parametrize("n,world", [(65536, 2), (65536, 8), (8192, 3), (5000, 8), (300, 4)])
def test_causal_query_shards_cover_rows_and_balance_work(n, world):
    shards = [q_shard(n, r, world, causal=True) for r in range(world)]
    assert shards[0].begin == 0 and shards[-1].end == n
    for a, b in zip(shards, shards[1:]):
        assert a.end == b.begin
    work = [s.end * (s.end + 1) / 2 - s.begin * (s.begin + 1) / 2 for s in shards]
    if n >= 256 * 4 * world:  # enough units to balance
        assert max(work) <= 1.25 * sum(work) / world
        equal = [q_shard(n, r, world) for r in range(world)]
        equal_work = [s.end * (s.end + 1) / 2 - s.begin * (s.begin + 1) / 2 for s in equal]
        assert max(work) < max(equal_work)


def test_shard_mode_switches_below_one_row_per_rank():
    assert shard_mode(8, 8) == "rows" and shard_mode(256, 8) == "rows"
    assert shard_mode(4, 8) == "queries" and shard_mode(1, 2) == "queries"


def _q_worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist

    from make_golden import make_inputs
    from oracle.attention import naive_attention

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n = 600
    q, k, v = (x.reshape(1, n, 64) for x in make_inputs((1, 1, n, 64), "normal", 5))
    assert shard_mode(1, world) == "queries"
    sh = q_shard(n, rank, world)
    # every rank holds the whole k and v; its query rows attend to all of them
    local = naive_attention(q[:, sh.begin:sh.end], k, v)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([sh.rows]))
    most = max(int(s.item()) for s in sizes)  # gloo gathers equal sizes: pad, then trim
    padded = torch.zeros((1, most, 64))
    padded[:, :sh.rows] = torch.from_numpy(np.ascontiguousarray(local)).float()
    pieces = [torch.zeros((1, most, 64)) for _ in sizes]
    dist.all_gather(pieces, padded)
    if rank == 0:
        full = torch.cat([p[:, :int(s.item())] for p, s in zip(pieces, sizes)], dim=1).numpy()
        want = naive_attention(q, k, v)
        result_q.put(float(np.max(np.abs(full - want))))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_query_sharded_forward_matches_full():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_q_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 0.0
