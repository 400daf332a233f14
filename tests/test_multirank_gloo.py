"""The multi-rank host plumbing of bench.py on CPU ranks (gloo, world size 2).

The GPU job shards batch rows across ranks with no data-path collective and
takes the slowest rank's time. Here each CPU rank runs the oracle on its shard
(the stand-in for its GPU's forward), the max-over-ranks reduction is checked,
and the gathered shards must equal the unsharded forward: rows never interact.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import layer as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = O.TransformerConfig(4, 24, 32, 2, 64, 1, True)
        params = O.init_params(cfg, 3)
        x, mask = O.generate_random_case(cfg, 4, 0.5, 1.0)
        lo, hi = bench.shard_rows(cfg.batch_size, world, rank, strong=True)
        sub = O.TransformerConfig(hi - lo, 24, 32, 2, 64, 1, True)
        out = O.baseline_forward(params, sub, x[lo:hi], mask[lo:hi])
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        slowest = bench.max_over_ranks([1.0 + rank, 5.0 - rank], dist, torch.device("cpu"))
        if rank == 0:
            full = O.baseline_forward(params, cfg, x, mask)
            torch.save({"full": full, "sharded": torch.cat(gathered), "max": slowest}, result_path)
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_and_reduce(tmp_path):
    world = 2
    path = str(tmp_path / "r.pt")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world,
                       start_method="spawn", join=True)
    r = torch.load(path)
    assert torch.equal(r["full"], r["sharded"])
    assert r["max"] == [2.0, 5.0]


def test_shard_rows_arithmetic():
    import bench

    assert bench.shard_rows(8, 4, 2, strong=True) == (4, 6)
    assert bench.shard_rows(8, 4, 3, strong=False) == (0, 8)
    with pytest.raises(ValueError, match="divisible"):
        bench.shard_rows(4, 8, 0, strong=True)


def _settle_worker(rank, world, port, result_path):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        count = [0]

        def step():
            # a step with a collective inside, as a tensor-parallel forward has
            t = torch.ones(3)
            dist.all_reduce(t)
            count[0] += 1

        # rank 1 would stop at once on its own clock, rank 0 only after 0.3 s
        bench.settle(step, 0.3 if rank == 0 else 0.0, dist, torch.device("cpu"))
        counts = torch.tensor([count[0]])
        gathered = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, counts)
        if rank == 0:
            torch.save([int(g.item()) for g in gathered], result_path)
    finally:
        dist.destroy_process_group()


def test_settle_runs_the_same_steps_on_every_rank(tmp_path):
    """bench.settle: ranks with different clocks still take the same number of
    steps, so the collectives inside the steps pair up."""
    path = str(tmp_path / "s.pt")
    mp.start_processes(_settle_worker, args=(2, _free_port(), path), nprocs=2,
                       start_method="spawn", join=True)
    counts = torch.load(path)
    assert counts[0] == counts[1] and counts[0] > 1


def _dropout_worker(rank, world, port, result_dir):
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)                       # one collective that everyone joins
    if rank == 1:
        # this rank leaves between steps, with nothing in flight
        with open(os.path.join(result_dir, "left"), "w") as f:
            f.write("1")
        os._exit(0)
    t0 = time.monotonic()
    err = ""
    try:
        dist.all_reduce(t)                   # its partner never joins this one
    except Exception as exc:  # noqa: BLE001 - any backend error ends the wait
        err = type(exc).__name__
    with open(os.path.join(result_dir, "rank0"), "w") as f:
        f.write(f"{err}\n{time.monotonic() - t0:.2f}")
    os._exit(0)


def test_rank_that_leaves_ends_the_next_collective_with_an_error(tmp_path):
    """Failure detection on the host: a rank that exits between steps makes the
    other rank's next collective end with an error within the process group's
    short timeout instead of waiting forever (no GPU involved)."""
    ctx = mp.start_processes(_dropout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                             start_method="spawn", join=False)
    import time

    deadline = time.monotonic() + 60
    while not ctx.join(timeout=1):
        assert time.monotonic() < deadline, "ranks did not finish"
    assert (tmp_path / "left").exists()
    err, secs = (tmp_path / "rank0").read_text().split("\n")
    assert err, "the surviving rank's collective must fail, not succeed"
    assert float(secs) < 30
