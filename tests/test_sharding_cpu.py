"""Multi-rank host logic on CPU: two gloo ranks in spawned processes.

* Each rank generates its own input shard from the counter-based generator
  (global element offsets); the shards concatenate to the one-shot stream, so
  the data a rank sees does not depend on the world size.
* The timed-region reduction returns the slowest rank's time on every rank.
* A rank that leaves between steps makes the next collective of the others
  fail with an error within the process-group timeout instead of hanging.
"""

import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from forgetune_b200 import sharding


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_cover_the_batch():
    for batch in (1, 7, 64, 65536, 65537):
        for world in (1, 2, 3, 8):
            blocks = [sharding.shard_rows(batch, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == batch
            for (a0, a1), (b0, b1) in zip(blocks, blocks[1:]):
                assert a1 == b0 and a0 <= a1
    with pytest.raises(ValueError):
        sharding.shard_rows(10, 2, 2)


def _rank_main(rank, world, port, out_dir, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from oracle import oracle
    sharding.init("gloo", timeout_s=10.0)
    try:
        if mode == "shards":
            rows, feats = 6, 5
            x = oracle.philox_normal(1, sharding.shard_element_offset(rank, rows, feats), rows * feats)
            slowest = sharding.max_over_ranks(1.5 + rank)
            sharding.barrier()
            np.save(os.path.join(out_dir, "shard%d.npy" % rank), x)
            np.save(os.path.join(out_dir, "max%d.npy" % rank), np.array([slowest]))
        elif mode == "lost_rank":
            sharding.barrier()
            if rank == 1:
                return  # leaves between steps, before the next collective
            t0 = time.time()
            try:
                sharding.max_over_ranks(1.0)
                outcome = "completed"
            except Exception as e:  # gloo raises on the missing peer
                outcome = "error:%s" % type(e).__name__
            with open(os.path.join(out_dir, "lost.txt"), "w") as f:
                f.write("%s %.1f" % (outcome, time.time() - t0))
    finally:
        try:
            import torch.distributed as dist
            if mode != "lost_rank":
                dist.destroy_process_group()
        except Exception:
            pass


def test_two_gloo_ranks_shard_and_reduce(tmp_path):
    mp.start_processes(_rank_main, args=(2, free_port(), str(tmp_path), "shards"), nprocs=2, join=True,
                       start_method="spawn")
    from oracle import oracle
    whole = oracle.philox_normal(1, 0, 2 * 6 * 5)
    got = np.concatenate([np.load(tmp_path / ("shard%d.npy" % r)) for r in range(2)])
    np.testing.assert_array_equal(got, whole)
    assert [float(np.load(tmp_path / ("max%d.npy" % r))[0]) for r in range(2)] == [2.5, 2.5]


def test_lost_rank_fails_the_next_collective(tmp_path):
    ctx = mp.start_processes(_rank_main, args=(2, free_port(), str(tmp_path), "lost_rank"), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.time() + 120
    while not ctx.join(timeout=5):
        assert time.time() < deadline, "ranks did not finish"
    outcome, secs = open(tmp_path / "lost.txt").read().split()
    assert outcome.startswith("error"), outcome
    assert float(secs) < 60
