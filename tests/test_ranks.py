"""Multi-process host logic on CPU (the reference's tests/test_serve_ranks.py:115-175 model): the replica dispatcher
(karpo_decision_b200.replicas) over loopback sockets with fake runners, and the bench's max-over-ranks aggregation
over real gloo process groups. No GPU: the runners are host functions; failures are made on the host (a runner that
raises, a process that exits, a process that never starts)."""

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
    """Sums the pack's ids after a delay (so requests overlap); a pack whose first id is -1 fails, and one whose first
    id is -2 makes a follower process exit at once (a replica that dies mid-stream)."""

    def __init__(self, rank: int) -> None:
        self.rank = rank

    def run(self, arrays):
        first = int(arrays["input_ids"][0])
        if first == -2 and self.rank != 0:
            os._exit(0)
        time.sleep(0.05)
        if first == -1:
            raise ValueError("bad pack")
        return np.array([[float(arrays["input_ids"].sum()), float(self.rank)]], dtype=np.float32)


def _dispatch_worker(rank: int, world: int, port: int, results, scenario: str) -> None:
    from concurrent.futures import wait

    from karpo_decision_b200 import replicas

    if rank != 0:
        if scenario == "absent" and rank == world - 1:
            return  # never connects: the dispatcher must give up waiting for it
        results[f"ran{rank}"] = replicas.serve(SlowRunner(rank), "127.0.0.1", port, rank)
        return
    dispatcher = replicas.Dispatcher(SlowRunner(0), world, "127.0.0.1", port, reply_timeout=30.0)
    if scenario == "absent":
        try:
            dispatcher.wait_ready(timeout=3.0)
        except TimeoutError as err:
            results["timeout"] = str(err)
        dispatcher.close()
        return
    dispatcher.wait_ready(timeout=60.0)
    if scenario == "crash":
        doomed = dispatcher.submit({"input_ids": np.array([-2, 0], dtype=np.int64)})
        if doomed.rank == 0:  # the local replica does not exit; the next pick is a follower
            doomed.result()
            doomed = dispatcher.submit({"input_ids": np.array([-2, 0], dtype=np.int64)})
        try:
            doomed.result(timeout=30)
        except replicas.ReplicaDown as err:
            results["down"] = (doomed.rank, str(err))
        after = [dispatcher.submit({"input_ids": np.arange(i, i + 4, dtype=np.int64)}) for i in range(12)]
        results["after_ranks"] = sorted({f.rank for f in after})
        results["after_ok"] = all(float(f.result(timeout=30)[0, 0]) == float(np.arange(i, i + 4).sum())
                                  for i, f in enumerate(after))
        results["stats"] = dispatcher.stats()
        dispatcher.close()
        return
    packs = [{"input_ids": np.arange(i, i + 10, dtype=np.int64), "cu": np.array([0, 10], dtype=np.int32)}
             for i in range(24)]
    start = time.perf_counter()
    futures = [dispatcher.submit(p) for p in packs]
    wait(futures)
    results["elapsed"] = time.perf_counter() - start
    results["correct"] = all(float(f.result()[0, 0]) == float(p["input_ids"].sum()) for f, p in zip(futures, packs))
    results["ranks_used"] = sorted({int(f.result()[0, 1]) for f in futures})
    results["routed_to"] = [f.rank for f in futures]
    errors = 0
    for _ in range(3):  # a failing pack comes back as an error; its follower keeps serving afterwards
        try:
            dispatcher.run({"input_ids": np.array([-1, 0], dtype=np.int64)})
        except (replicas.ReplicaError, ValueError):
            errors += 1
    results["errors"] = errors
    results["after_error"] = float(dispatcher.run({"input_ids": np.arange(5, dtype=np.int64)})[0, 0])
    results["stats"] = dispatcher.stats()
    dispatcher.close()


def _run(world: int, scenario: str) -> dict:
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_dispatch_worker, args=(world, _free_port(), results, scenario), nprocs=world, join=True)
        return dict(results)


def test_dispatcher_spreads_packs_over_replicas_and_survives_a_failing_pack():
    r = _run(3, "spread")
    assert r["correct"]
    assert r["ranks_used"] == [0, 1, 2]
    # fewest in flight, ties in turn: 24 packs queued at once go round the three replicas
    assert r["routed_to"][:6] == [0, 1, 2, 0, 1, 2]
    stats = r["stats"]
    assert sum(stats["served"]) + sum(stats["failed"]) == 24 + 3 + 1 and sum(stats["failed"]) == 3
    assert stats["served"][1] + stats["failed"][1] == r["ran1"] and stats["served"][2] + stats["failed"][2] == r["ran2"]
    # 24 packs of 50 ms on 3 replicas overlap: well under the 1.2 s one replica would take
    assert r["elapsed"] < 0.9
    assert r["errors"] == 3 and r["after_error"] == 10.0
    assert all(ms >= 0.0 for ms in stats["handover_ms"])


def test_a_replica_that_exits_is_marked_down_and_skipped():
    """A follower process that dies mid-pack (its connection closes) fails that pack with ReplicaDown at once; later
    packs go to the replicas still serving."""
    r = _run(3, "crash")
    rank, message = r["down"]
    assert rank in (1, 2) and "connection" in message
    assert rank not in r["after_ranks"] and r["after_ok"]
    assert r["stats"]["down"][rank] is not None


def test_waiting_for_a_replica_that_never_starts_times_out():
    r = _run(3, "absent")
    assert "never reported ready" in r["timeout"]


def test_pack_wire_format_round_trips():
    from karpo_decision_b200.replicas import decode, encode

    arrays = {"input_ids": np.arange(7, dtype=np.int64), "cu": np.array([0, 3, 7], dtype=np.int32),
              "x": np.ones((2, 3), dtype=np.float32), "empty": np.zeros(0, dtype=np.int16)}
    back = decode(encode(arrays))
    assert list(back) == list(arrays)
    for k in arrays:
        assert back[k].dtype == arrays[k].dtype and np.array_equal(back[k], arrays[k])


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
