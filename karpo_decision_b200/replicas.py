"""Replica serving across GPUs: one full model per GPU, one process per GPU, and a dispatcher in the first process
that sends each pack to the replica with the fewest packs in flight, ties taken in turn. That routing policy is the
reference's multi-GPU scheme (serve/server.py:203-239); the packed forward itself exchanges nothing between GPUs, so no
collective touches the data path.

Design of this module:
- Transport: one TCP connection per follower to the dispatcher, carrying length-prefixed frames. A pack travels as
  its host arrays' raw bytes behind a small JSON header (names, dtypes, shapes), a reply as the raw float32 logits;
  nothing is pickled, so a follower never unpickles what it receives.
- Queues: the dispatcher keeps one host queue per replica (its own GPU included) drained by one thread per replica;
  ``submit`` picks the replica at arrival and returns a ``concurrent.futures.Future`` for the reply.
- Failures: a pack that raises on a follower comes back as an error frame, the future raises ``ReplicaError`` and the
  follower keeps serving. A follower whose connection closes (the process exited) or that does not reply within the
  reply timeout is marked down: its pending packs fail at once and no pack is routed to it again.

Use: every follower calls ``serve(runner, host, port, rank)``; the dispatcher process builds
``Dispatcher(local_runner, world, host, port)``, calls ``wait_ready()``, then ``submit`` / ``run`` from any number of
threads, and ``close()`` at the end. A runner is any object with ``run(arrays) -> np.ndarray`` (``PackRunner`` runs
the B200 forward and readout on this process's GPU).
"""

from __future__ import annotations

import json
import queue
import socket
import struct
import threading
import time
from concurrent.futures import Future
from typing import Any, Protocol

import numpy as np

__all__ = ["Dispatcher", "PackRunner", "ReplicaError", "ReplicaDown", "decode", "encode", "serve"]

# frame: magic, kind, sequence number, payload length
_FRAME = struct.Struct("<2sBxIQ")
_MAGIC = b"KD"
HELLO, JOB, REPLY, ERROR, STOP = 1, 2, 3, 4, 5


class Runner(Protocol):
    def run(self, arrays: dict[str, np.ndarray]) -> np.ndarray: ...


class ReplicaError(RuntimeError):
    """A pack failed on a follower; the follower is still serving."""


class ReplicaDown(RuntimeError):
    """A follower's connection closed or it stopped replying; it receives no more packs."""


def encode(arrays: dict[str, Any]) -> bytes:
    """Host arrays as one byte string: a JSON header of (name, dtype, shape), then each array's raw bytes in order."""
    items = [(k, np.ascontiguousarray(v)) for k, v in arrays.items()]
    header = json.dumps([[k, v.dtype.str, list(v.shape)] for k, v in items]).encode()
    return b"".join([struct.pack("<I", len(header)), header, *(v.tobytes() for _, v in items)])


def decode(blob: bytes) -> dict[str, np.ndarray]:
    """The arrays of ``encode``'s byte string (copies, so they own their memory)."""
    (n,) = struct.unpack_from("<I", blob)
    at = 4 + n
    out = {}
    for name, dtype, shape in json.loads(blob[4:at]):
        dt = np.dtype(dtype)
        count = int(np.prod(shape, dtype=np.int64))
        out[name] = np.frombuffer(blob, dt, count, at).reshape(shape).copy()
        at += count * dt.itemsize
    return out


def _send(sock: socket.socket, kind: int, seq: int, payload: bytes = b"") -> None:
    sock.sendall(_FRAME.pack(_MAGIC, kind, seq, len(payload)) + payload)


def _read_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray(n)
    view, got = memoryview(buf), 0
    while got < n:
        k = sock.recv_into(view[got:], n - got)
        if k == 0:
            raise ConnectionError("connection closed")
        got += k
    return bytes(buf)


def _receive(sock: socket.socket) -> tuple[int, int, bytes]:
    magic, kind, seq, length = _FRAME.unpack(_read_exact(sock, _FRAME.size))
    if magic != _MAGIC:
        raise ConnectionError("not a replica frame")
    return kind, seq, _read_exact(sock, length) if length else b""


class PackRunner:
    """Runs one pack at a time on this process's GPU: host arrays -> pinned -> device -> ``model`` -> ``head`` ->
    host logits (float32, markers x codes)."""

    def __init__(self, model: Any, head: Any, device: Any) -> None:
        self.model, self.head, self.device = model, head, device
        self.lock = threading.Lock()

    def run(self, arrays: dict[str, np.ndarray]) -> np.ndarray:
        import torch

        from .pack import from_arrays

        with self.lock:
            torch.cuda.set_device(self.device)
            logits = self.head(self.model(from_arrays(arrays, self.device, pinned=True)))
            return logits.float().cpu().numpy()


def serve(runner: Runner, host: str, port: int, rank: int, connect_timeout: float = 120.0) -> int:
    """A follower: connects to the dispatcher, reports ready, then runs every pack it is sent until told to stop (or
    the dispatcher goes away); returns the number of packs it ran."""
    deadline = time.monotonic() + connect_timeout
    while True:
        try:
            sock = socket.create_connection((host, port), timeout=5.0)
            break
        except OSError:
            if time.monotonic() > deadline:
                raise
            time.sleep(0.05)
    sock.settimeout(None)
    sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    ran = 0
    with sock:
        _send(sock, HELLO, rank)
        while True:
            try:
                kind, seq, payload = _receive(sock)
            except ConnectionError:
                return ran
            if kind == STOP:
                return ran
            if kind != JOB:
                continue
            try:
                logits = np.ascontiguousarray(runner.run(decode(payload)), dtype=np.float32)
                reply = (REPLY, encode({"logits": logits}))
            except Exception as err:  # the pack's failure goes back to the dispatcher; this follower serves on
                reply = (ERROR, f"{type(err).__name__}: {err}".encode())
            ran += 1
            _send(sock, reply[0], seq, reply[1])


class _Slot:
    """One replica as the dispatcher sees it: its queue, counters and (for followers) its connection."""

    def __init__(self, rank: int) -> None:
        self.rank = rank
        self.queue: queue.Queue = queue.Queue()
        self.in_flight = 0  # queued + running
        self.served = 0
        self.failed = 0
        self.busy_s = 0.0
        self.send_ms: list[float] = []
        self.down: str | None = None
        self.sock: socket.socket | None = None
        self.thread: threading.Thread | None = None


class Dispatcher:
    """Routes packs to the replica with the fewest in flight (slot 0 is this process's own ``local`` runner, slot r
    the follower of rank r), ties taken in turn from the slot after the last one picked."""

    def __init__(self, local: Runner | None, world: int, host: str = "127.0.0.1", port: int = 0,
                 reply_timeout: float = 600.0) -> None:
        self.local, self.world, self.reply_timeout = local, world, reply_timeout
        self.slots = [_Slot(r) for r in range(world)]
        if local is None:
            self.slots[0].down = "no local runner"
        self.lock = threading.Lock()
        self.turn = 0
        self.listener = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.listener.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.listener.bind((host, port))
        self.listener.listen(max(world, 1))
        self.port = self.listener.getsockname()[1]
        self._stopped = False

    # ---------------------------------------------------------------------------------------------- set-up
    def wait_ready(self, timeout: float = 600.0) -> None:
        """Accepts every follower's connection and ready report (raises TimeoutError if one is missing), then starts
        one worker thread per replica."""
        self.listener.settimeout(timeout)
        pending = self.world - 1
        deadline = time.monotonic() + timeout
        while pending:
            self.listener.settimeout(max(deadline - time.monotonic(), 0.001))
            try:
                sock, _ = self.listener.accept()
            except TimeoutError as err:
                raise TimeoutError(f"{pending} follower(s) never reported ready") from err
            sock.settimeout(max(deadline - time.monotonic(), 0.001))
            kind, rank, _ = _receive(sock)
            if kind != HELLO or not 0 < rank < self.world or self.slots[rank].sock is not None:
                sock.close()
                continue
            sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            sock.settimeout(self.reply_timeout)
            self.slots[rank].sock = sock
            pending -= 1
        for slot in self.slots:
            slot.thread = threading.Thread(target=self._drain, args=(slot,), daemon=True,
                                           name=f"replica-{slot.rank}")
            slot.thread.start()

    # ---------------------------------------------------------------------------------------------- routing
    def pick(self) -> _Slot:
        with self.lock:
            live = [s for s in self.slots if s.down is None]
            if not live:
                raise ReplicaDown("no replica is serving")
            n = self.world
            slot = min(live, key=lambda s: (s.in_flight, (s.rank - self.turn) % n))
            slot.in_flight += 1
            self.turn = (slot.rank + 1) % n
            return slot

    def submit(self, arrays: dict[str, np.ndarray]) -> Future:
        """Queues ``arrays`` on the least loaded replica; the future's result is the pack's logits."""
        future: Future = Future()
        future.submitted = time.perf_counter()
        slot = self.pick()
        future.rank = slot.rank
        slot.queue.put((arrays, future))
        return future

    def run(self, arrays: dict[str, np.ndarray]) -> np.ndarray:
        return self.submit(arrays).result()

    # ---------------------------------------------------------------------------------------------- workers
    def _finish(self, slot: _Slot, future: Future, result=None, error: BaseException | None = None) -> None:
        with self.lock:
            slot.in_flight -= 1
            if error is None:
                slot.served += 1
            else:
                slot.failed += 1
        future.finished = time.perf_counter()
        if error is None:
            future.set_result(result)
        else:
            future.set_exception(error)

    def _mark_down(self, slot: _Slot, why: str) -> None:
        with self.lock:
            slot.down = why
        while True:  # packs still queued there fail now rather than wait on a replica that is gone
            try:
                item = slot.queue.get_nowait()
            except queue.Empty:
                return
            if item is not None:
                self._finish(slot, item[1], error=ReplicaDown(f"replica {slot.rank}: {why}"))

    def _drain(self, slot: _Slot) -> None:
        seq = 0
        while True:
            item = slot.queue.get()
            if item is None:
                if slot.sock is not None and slot.down is None:
                    try:
                        _send(slot.sock, STOP, 0)
                    except OSError:
                        pass
                return
            arrays, future = item
            if slot.down is not None:
                self._finish(slot, future, error=ReplicaDown(f"replica {slot.rank}: {slot.down}"))
                continue
            start = time.perf_counter()
            if slot.rank == 0:
                try:
                    result = self.local.run(arrays)
                except Exception as err:
                    self._finish(slot, future, error=err)
                else:
                    slot.busy_s += time.perf_counter() - start
                    self._finish(slot, future, result)
                continue
            seq += 1
            try:
                _send(slot.sock, JOB, seq, encode(arrays))
                slot.send_ms.append((time.perf_counter() - start) * 1000.0)
                kind, got, payload = _receive(slot.sock)
            except (OSError, ConnectionError) as err:
                why = "no reply within the timeout" if isinstance(err, TimeoutError) else f"connection lost ({err})"
                self._finish(slot, future, error=ReplicaDown(f"replica {slot.rank}: {why}"))
                self._mark_down(slot, why)
                continue
            slot.busy_s += time.perf_counter() - start
            if kind == REPLY and got == seq:
                self._finish(slot, future, decode(payload)["logits"])
            else:
                self._finish(slot, future, error=ReplicaError(f"replica {slot.rank}: {payload.decode(errors='replace')}"))

    # ---------------------------------------------------------------------------------------------- end
    def close(self) -> None:
        """Stops every follower (after the packs already queued) and the worker threads."""
        if self._stopped:
            return
        self._stopped = True
        for slot in self.slots:
            slot.queue.put(None)
        for slot in self.slots:
            if slot.thread is not None:
                slot.thread.join()
            if slot.sock is not None:
                slot.sock.close()
        self.listener.close()

    def stats(self) -> dict:
        """Per replica: packs served and failed, busy seconds, mean milliseconds to hand a pack over."""
        return {"served": [s.served for s in self.slots], "failed": [s.failed for s in self.slots],
                "busy_s": [round(s.busy_s, 4) for s in self.slots],
                "handover_ms": [round(float(np.mean(s.send_ms)), 4) if s.send_ms else 0.0 for s in self.slots],
                "down": [s.down for s in self.slots]}
