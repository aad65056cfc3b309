"""Replica serving across GPUs, the reference's multi-GPU scheme (serve/server.py:161-266): one full model per GPU
(one process per rank under torchrun), rank 0 routing each pack to the rank with the fewest packs in flight (itself
included, ties in turn), packs and replies handed over on the CPU through two-member gloo groups. The packed forward
itself exchanges nothing between GPUs, so no collective touches the data path.

A rank other than 0 runs ``follow``; rank 0 builds a ``Router`` and calls ``Router.run(arrays)`` from as many threads
as it serves concurrently. A pack is its host arrays (``synthetic_pack_arrays`` layout); a reply is the pack's readout
logits (numpy float32, markers x codes). A failing pack on a follower comes back as an error and the follower keeps
serving (serve/server.py:252-266); rank 0 raises it to its caller.
"""

from __future__ import annotations

import threading
import time
from typing import Any, Protocol

import numpy as np
import torch
import torch.distributed as dist

STOP = "stop"
READY = "ready"


class Runner(Protocol):
    def run(self, arrays: dict[str, np.ndarray]) -> np.ndarray: ...


class PackRunner:
    """Runs one pack at a time on this rank's GPU: pinned host arrays -> device -> ``model`` -> ``head`` -> host."""

    def __init__(self, model: Any, head: Any, device: torch.device) -> None:
        self.model, self.head, self.device = model, head, device
        self.lock = threading.Lock()

    def run(self, arrays: dict[str, np.ndarray]) -> np.ndarray:
        from .pack import from_arrays

        with self.lock:
            torch.cuda.set_device(self.device)
            logits = self.head(self.model(from_arrays(arrays, self.device, pinned=True)))
            return logits.float().cpu().numpy()


class Link:
    """Rank 0's line to rank ``rank``: a two-member group, one message at a time."""

    def __init__(self, group: Any, rank: int) -> None:
        self.group, self.rank = group, rank
        self.lock = threading.Lock()

    def send(self, message: Any) -> None:
        dist.broadcast_object_list([message], src=0, group=self.group)

    def receive(self) -> Any:
        box: list[Any] = [None]
        dist.broadcast_object_list(box, src=self.rank, group=self.group)
        return box[0]

    def call(self, message: Any) -> tuple[Any, float]:
        """The rank's reply and the milliseconds spent handing the message over."""
        with self.lock:
            start = time.perf_counter()
            self.send(message)
            handed = (time.perf_counter() - start) * 1000.0
            return self.receive(), handed


class Router:
    """Routes packs to the rank with the fewest in flight (slot 0 is rank 0's own runner), ties in turn."""

    def __init__(self, runner: Runner, links: list[Link]) -> None:
        self.runner, self.links = runner, links
        self.in_flight = [0] * (len(links) + 1)
        self.next = 0
        self.served = [0] * (len(links) + 1)
        self.lock = threading.Lock()

    def pick(self) -> int:
        with self.lock:
            n = len(self.in_flight)
            slot = min(range(n), key=lambda r: (self.in_flight[r], (r - self.next) % n))
            self.in_flight[slot] += 1
            self.next = (slot + 1) % n
            return slot

    def done(self, slot: int) -> None:
        with self.lock:
            self.in_flight[slot] -= 1
            self.served[slot] += 1

    def run(self, arrays: dict[str, np.ndarray]) -> np.ndarray:
        slot = self.pick()
        try:
            if slot == 0:
                return self.runner.run(arrays)
            (reply, error), _ = self.links[slot - 1].call(arrays)
            if error is not None:
                raise RuntimeError(f"rank {slot}: {error[0]}: {error[1]}")
            return reply
        finally:
            self.done(slot)

    def ready(self) -> None:
        """Returns once every other rank has loaded its model."""
        for link in self.links:
            link.receive()

    def stop(self) -> None:
        for link in self.links:
            with link.lock:
                link.send(STOP)


def links(world_size: int) -> list[Link]:
    """Rank 0's links; every rank must call ``groups`` first (collective group creation)."""
    return [Link(group, rank) for rank, group in enumerate(groups(world_size)) if rank > 0]


_GROUPS: list[Any] = []


def groups(world_size: int) -> list[Any]:
    """The two-member groups {0, k} for k = 1 .. world_size - 1 (index k; index 0 unused), created once on every
    rank in the same order."""
    if not _GROUPS:
        _GROUPS.append(None)
        for rank in range(1, world_size):
            _GROUPS.append(dist.new_group([0, rank]))
    return _GROUPS


def follow(runner: Runner, rank: int, world_size: int) -> int:
    """A rank other than 0: reports ready, then runs what rank 0 hands it until STOP; returns the packs it ran."""
    group = groups(world_size)[rank]
    dist.broadcast_object_list([READY], src=rank, group=group)
    served = 0
    while True:
        box: list[Any] = [None]
        dist.broadcast_object_list(box, src=0, group=group)
        if isinstance(box[0], str) and box[0] == STOP:
            return served
        try:
            reply = (runner.run(box[0]), None)
        except Exception as error:  # noqa: BLE001 - rank 0 answers for it; this rank keeps following
            reply = (None, (type(error).__name__, str(error)))
        served += 1
        dist.broadcast_object_list([reply], src=rank, group=group)
