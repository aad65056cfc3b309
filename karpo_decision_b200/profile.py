"""Per-kernel CUDA-event timing of libkd_b200 launches (used by bench.py): while ``kernels()`` is active, every entry
point call records an event before and after its launch on the current stream, so each kernel's device time, launch
count and share are measured inside the timed region itself."""

from __future__ import annotations

import contextlib
from collections import defaultdict

import torch

from . import _lib

#: Argument positions of (M, N, K) in the GEMM entry points.
_GEMM_MNK = {"kd_gemm_bf16": (8, 9, 10), "kd_gemm_fp8": (10, 11, 12), "kd_qkv_projection": (4, 5, 6),
             "kd_qkv_projection_fp8": (6, 7, 8)}


class KernelTimes:
    def __init__(self) -> None:
        self.records: list[tuple[str, torch.cuda.Event, torch.cuda.Event, float]] = []

    def before(self, name: str, args: tuple):
        start = torch.cuda.Event(enable_timing=True)
        start.record()
        return start

    def after(self, name: str, args: tuple, start) -> None:
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        flops = 0.0
        if name in _GEMM_MNK:
            m, n, k = (args[i] for i in _GEMM_MNK[name])
            flops = 2.0 * m * n * k
        self.records.append((name, start, end, flops))

    @property
    def launches(self) -> int:
        return len(self.records)

    def times(self) -> dict[str, list[tuple[float, float]]]:
        """Per entry point, each launch's (device milliseconds, FLOPs) in launch order."""
        torch.cuda.synchronize()
        out: dict[str, list[tuple[float, float]]] = defaultdict(list)
        for name, start, end, flops in self.records:
            out[name].append((start.elapsed_time(end), flops))
        return out

    def summary(self, prefix: str) -> dict:
        """Launch count, mean device ms and mean FLOPs per launch of the kernels whose name contains ``prefix``."""
        rows = [r for name, rs in self.times().items() if prefix in name for r in rs]
        if not rows:
            return {"launches": 0, "mean_ms": None, "flops_per_launch": 0.0}
        total_ms = sum(ms for ms, _ in rows)
        return {"launches": len(rows), "mean_ms": total_ms / len(rows),
                "flops_per_launch": sum(f for _, f in rows) / len(rows)}

    def shares(self) -> dict:
        times = self.times()
        total = sum(ms for rs in times.values() for ms, _ in rs) or 1.0
        return {name: {"launches": len(rs), "ms": round(sum(ms for ms, _ in rs), 4),
                       "share": round(sum(ms for ms, _ in rs) / total, 4)} for name, rs in sorted(times.items())}


@contextlib.contextmanager
def kernels(stream: torch.cuda.Stream | None = None):
    prof = KernelTimes()
    _lib.set_profiler(prof)
    try:
        with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
            yield prof
    finally:
        _lib.set_profiler(None)
