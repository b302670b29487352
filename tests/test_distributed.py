"""Head / rollout sharding host logic, on CPU with world-size-2 gloo ranks."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cast_b200 import distributed as cd


def test_head_range_partitions_heads():
    for world in (1, 2, 4, 8):
        ranges = [cd.head_range(24, world, r) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == 24
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert len({hi - lo for lo, hi in ranges}) == 1
    with pytest.raises(ValueError):
        cd.head_range(24, 5, 0)
    with pytest.raises(ValueError):
        cd.head_range(24, 2, 2)


def test_gather_heads_single_rank_is_identity():
    x = torch.randn(2, 6, 5, 4).bfloat16()
    assert torch.equal(cd.gather_heads(x, 1), x)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ok = []
        for b in (1, 2):
            full = torch.arange(b * 8 * 3 * 4, dtype=torch.float32).reshape(b, 8, 3, 4).bfloat16()
            lo, hi = cd.head_range(8, world, rank)
            got = cd.gather_heads(full[:, lo:hi].clone(), world)
            ok.append(bool(torch.equal(got, full)))
        # the bench's max-over-ranks timing reduction
        t = torch.tensor([1.0 + rank, 5.0 - rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok.append(t.tolist() == [float(world), 5.0])
        with open(os.path.join(result_dir, f"r{rank}"), "w") as fh:
            fh.write(",".join(str(int(v)) for v in ok))
    finally:
        dist.destroy_process_group()


def test_gather_heads_two_gloo_ranks(tmp_path):
    world = 2
    mp.get_context("spawn")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        assert (tmp_path / f"r{r}").read_text() == "1,1,1"
