"""Multi-rank host logic on CPU (gloo, world size 2): batch sharding with
replicated weights gives the full-batch result, and the timing reduction is a
max over ranks.  The per-rank compute here is the CPU oracle standing in for
the GPU kernel (no GPU is needed to test the sharding logic)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from complex_conv2d.distributed import batch_shard


def test_batch_shard_even_and_uneven():
    assert [batch_shard(64, 8, r) for r in range(8)] == [(8 * r, 8) for r in range(8)]
    parts = [batch_shard(10, 4, r) for r in range(4)]
    assert parts == [(0, 3), (3, 3), (6, 2), (8, 2)]
    assert sum(c for _, c in parts) == 10
    assert batch_shard(3, 4, 3) == (3, 0)
    with pytest.raises(ValueError):
        batch_shard(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, global_batch, result_path):
    import torch.distributed as dist

    import oracle
    from complex_conv2d.distributed import batch_shard, gather_batch, max_over_ranks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = oracle.ConvCase(global_batch, 8, 9, 9, 12, 3, 3, 1, 1, 1, 1)
        x, wr, wi = oracle.make_inputs(case, input_seed=3)  # same seed: replicated data/weights
        start, count = batch_shard(global_batch, world, rank)
        y_local = oracle.four_conv(x[start:start + count], wr, wi, (1, 1), (1, 1),
                                   dtype=torch.float32)
        y_all = gather_batch(y_local, global_batch)
        t = max_over_ranks(float(rank + 1))
        if rank == 0:
            ref = oracle.four_conv(x, wr, wi, (1, 1), (1, 1), dtype=torch.float32)
            torch.save({"ok": bool(torch.equal(y_all, ref)), "t": t, "shape": tuple(y_all.shape)},
                       result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("global_batch", [4, 5])
def test_two_rank_sharded_forward_matches_full_batch(tmp_path, global_batch):
    path = str(tmp_path / "res.pt")
    mp.spawn(_worker, args=(2, _free_port(), global_batch, path), nprocs=2, join=True)
    res = torch.load(path)
    assert res["ok"], res
    assert res["t"] == 2.0
    assert res["shape"][0] == global_batch
