"""World-size-2 gloo ranks on the CPU: request sharding of batch messages (no
data-path collective) and the max-over-ranks timing reduction the benchmark
uses."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from longspark_b200.requests import BATCH_FORMAT, owner_rank, split_batch_message
        ids = [f"r{i}" for i in range(9)]
        counts = [(i % 4) + 1 for i in range(9)]
        keys = torch.arange(sum(counts), dtype=torch.float32).view(1, -1, 1, 1).expand(2, -1, 1, 4).contiguous()
        msg = dict(format=BATCH_FORMAT, ids=ids, lengths=[100 + c for c in counts], commit_lens=counts,
                   export_counts=counts, keys=keys, values=keys.clone(), last_hidden=torch.zeros(9, 2, 8))
        mine = split_batch_message(msg, world, rank)
        assert all(owner_rank(i, world) == rank for i in mine["ids"])
        # every request lands on exactly one rank
        n = torch.tensor([len(mine["ids"])])
        dist.all_reduce(n)
        rows = torch.tensor([mine["keys"].shape[1]])
        dist.all_reduce(rows)
        # max-over-ranks timing as in bench.dist_max
        t = torch.tensor([1.0 + rank])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[rank] = (int(n.item()), int(rows.item()), float(t.item()))
    finally:
        dist.destroy_process_group()


def test_two_rank_request_sharding():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    assert res[0] == res[1] == (9, sum((i % 4) + 1 for i in range(9)), 2.0)
