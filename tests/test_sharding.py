"""Multi-GPU partitioning, exercised without a GPU: the assignment functions and a
2-rank gloo all-gather of per-rank outputs (the one collective of the path)."""

import os
import socket

import torch
import torch.multiprocessing as mp

from mzoo_b200 import sharding


def test_shard_sequences_covers_and_balances():
    g = torch.Generator().manual_seed(1)
    lens = torch.randint(8192, 131073, (128,), generator=g).tolist()
    for world in (1, 2, 4, 8):
        parts = sharding.shard_sequences(lens, world)
        assert sorted(b for p in parts for b in p) == list(range(128))
        loads = [sum(lens[b] for b in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)  # greedy LPT bound


def test_shard_tokens_cyclic():
    parts = sharding.shard_tokens(1000, 3, chunk=128)
    assert sorted(t for p in parts for t in p) == list(range(1000))
    assert parts[0][:128] == list(range(128)) and parts[1][0] == 128 and parts[0][128] == 384


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lens = list(range(10, 0, -1)) + [3, 7]
    parts = sharding.shard_sequences(lens, world)
    mine = parts[rank]
    # each rank "computes" row b = b * [1, 2, 3] for the units it owns
    local = torch.stack([torch.tensor([1.0, 2.0, 3.0]) * b for b in mine])
    full = sharding.gather_rows(local, mine, parts)
    # the bench's timing reduction: every rank reports the slowest rank's time
    import bench
    slowest = bench.max_over_ranks(torch, dist, 1.5 + rank, torch.device("cpu"))
    q.put((rank, full.tolist(), slowest))
    dist.barrier()
    dist.destroy_process_group()


def test_gather_rows_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = [[1.0 * b, 2.0 * b, 3.0 * b] for b in range(12)]
    for _, full, slowest in results:
        assert full == expect
        assert slowest == 2.5
