"""Multi-process host logic on CPU with real gloo process groups over loopback (the reference's
tests/test_serve_ranks.py:115-175 model): the replica router (karpo_decision_b200.replicas) with fake runners, and
the bench's max-over-ranks aggregation. No GPU: the runners are host functions; failures are made on the host."""

import os
import socket
import time

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class SlowRunner:
    """Sums the pack's ids after a delay (so requests overlap); a pack whose first id is -1 fails."""

    def __init__(self, rank: int) -> None:
        self.rank = rank

    def run(self, arrays):
        time.sleep(0.05)
        if int(arrays["input_ids"][0]) == -1:
            raise ValueError("bad pack")
        return np.array([[float(arrays["input_ids"].sum()), float(self.rank)]], dtype=np.float32)


def _router_worker(rank: int, world: int, port: int, results) -> None:
    import threading

    from karpo_decision_b200 import replicas

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    runner = SlowRunner(rank)
    if rank != 0:
        results[f"served{rank}"] = replicas.follow(runner, rank, world)
        dist.destroy_process_group()
        return
    router = replicas.Router(runner, replicas.links(world))
    router.ready()
    packs = [{"input_ids": np.arange(i, i + 10, dtype=np.int64)} for i in range(24)]
    out = [None] * len(packs)

    def work(i):
        out[i] = router.run(packs[i])

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(packs))]
    start = time.perf_counter()
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    results["elapsed"] = time.perf_counter() - start
    results["correct"] = all(float(out[i][0, 0]) == float(packs[i]["input_ids"].sum()) for i in range(len(packs)))
    results["ranks_used"] = sorted({int(o[0, 1]) for o in out})
    # a failing pack comes back as an error; the follower keeps serving afterwards
    errors = 0
    for _ in range(3):
        try:
            router.run({"input_ids": np.array([-1, 0], dtype=np.int64)})
        except (RuntimeError, ValueError):
            errors += 1
    results["errors"] = errors
    results["after_error"] = float(router.run({"input_ids": np.arange(5, dtype=np.int64)})[0, 0])
    results["served0"] = router.served[0]  # rank 0's own runs; followers count theirs
    results["routed"] = sum(router.served)
    router.stop()
    dist.destroy_process_group()


def test_router_spreads_packs_over_ranks_and_survives_a_failing_pack():
    world = 3
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_router_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        r = dict(results)
    assert r["correct"]
    assert r["ranks_used"] == [0, 1, 2]
    assert r["routed"] == 24 + 3 + 1
    assert r["served0"] + r["served1"] + r["served2"] == r["routed"]
    # 24 packs of 50 ms on 3 ranks overlap: well under the 1.2 s one rank would take
    assert r["elapsed"] < 0.9
    assert r["errors"] == 3 and r["after_error"] == 10.0


def _aggregate_worker(rank: int, world: int, port: int, results) -> None:
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ms, e2e_ms, value, e2e_value = bench.aggregate([10.0 * (rank + 1), 20.0 + rank], 1000, world, "cpu", dist)
    results[rank] = (ms, e2e_ms, value, e2e_value)
    dist.destroy_process_group()


def test_bench_takes_the_slowest_rank():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_aggregate_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        r = dict(results)
    for rank in range(world):
        ms, e2e_ms, value, e2e_value = r[rank]
        assert ms == 20.0 and e2e_ms == 21.0
        assert value == pytest.approx(1000 * 2 / 0.020) and e2e_value == pytest.approx(1000 * 2 / 0.021)
