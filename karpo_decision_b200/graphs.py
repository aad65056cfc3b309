"""CUDA graphs of the packed forward per bucketed pack size: the B200 counterpart of the reference's ``--graphs``
path (serve/graphs.py:54-132 for Gemma, serve/qwen_graphs.py:64-197 for Qwen3.5), which removes the per-kernel launch
cost of small packs.

Every kernel of the body reads the sequence boundaries from device memory and allocates nothing, so one graph per
bucket of B tokens serves any pack of at most B tokens, whatever its sequences:
- the pack's ids and positions are copied into the bucket's static buffers;
- the rows past the pack become padding sequences of at most ``PAD_SEQUENCE`` tokens each, computed and never read;
- the boundary slots past them are empty sequences, so the attention grid of the capture stays valid.
The reference instead captures one right-padded single-sequence (Gemma) or per-segment (Qwen) layout per bucket. As in
the reference, the head (a bidirectional model's last layer at the markers, then the final norm) runs after the replay
on the real rows, outside the graph (serve/qwen_graphs.py:160-167, serve/graphs.py:114-118). Packs
no bucket covers, and branched block layouts (their virtual sequences are planned per pack), run the plain path of
the same kernels (serve/graphs.py:121-132).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from .pack import Pack
from .packed import Packed

#: Padding rows form sequences of at most this many tokens (their causal attention stays cheap).
PAD_SEQUENCE = 256
#: Bucket bands as (step, top): sizes step, 2 step, ... up to top, the step doubling from band to band, so a pack is
#: padded by at most 64 tokens up to 2,048 and by at most a sixteenth of its size beyond. The reference's fine
#: buckets, the ones its fast Qwen path captures (serve/qwen_graphs.py:171).
FINE_BANDS = ((64, 2048), (128, 4096), (256, 8192), (512, 16384), (1024, 32768), (2048, 65536))


def fine_buckets(max_tokens: int) -> tuple[int, ...]:
    """The fine buckets up to the first one holding ``max_tokens`` tokens (at most 65,536)."""
    if not 0 < max_tokens <= FINE_BANDS[-1][1]:
        raise ValueError(f"max_tokens must be in [1, {FINE_BANDS[-1][1]}]")
    out: list[int] = []
    low = 0
    for step, top in FINE_BANDS:
        size = low + step
        while size <= top:
            out.append(size)
            if size >= max_tokens:
                return tuple(out)
            size += step
        low = top
    return tuple(out)


#: Default buckets: the fine buckets up to 65,536 tokens (112 graphs, captured at construction; they share one
#: workspace, so their cost is capture time, not memory).
DEFAULT_BUCKETS = fine_buckets(65536)


@dataclass
class _Bucket:
    size: int
    ids: torch.Tensor  # (size,) int64
    seqpos: torch.Tensor  # (size,) int64
    cu: torch.Tensor  # (slots + 1,) int32
    pack: Pack
    graph: torch.cuda.CUDAGraph
    out: torch.Tensor  # the body's output rows (size, hidden)
    keep: tuple  # tensors the graph reads (workspace, rotary tables): held while the graph lives


class Graphs:
    """Captured bodies of ``model`` for the given pack sizes; call it like the model: ``graphs(pack) -> (M, hidden)``.

    ``max_sequences`` bounds the real sequences of a covered pack. Capture runs at construction, from the largest
    bucket down (the reference's order, serve/graphs.py:94-98), after one eager warm-up per bucket."""

    def __init__(self, model: Packed, buckets: tuple[int, ...] = DEFAULT_BUCKETS, max_sequences: int = 512) -> None:
        self.model = model
        self.device = model.device
        self.max_sequences = max_sequences
        self.buckets: list[_Bucket] = []
        sizes = sorted(set(int(b) for b in buckets), reverse=True)
        if not sizes:
            raise ValueError("at least one bucket is needed")
        self.pool = torch.cuda.graph_pool_handle()
        model.workspace(sizes[0])  # one workspace at the largest bucket, shared by every graph
        for size in sizes:
            self.buckets.append(self._capture(size))
        self.buckets.sort(key=lambda b: b.size)

    def _slots(self, size: int) -> int:
        return self.max_sequences + -(-size // PAD_SEQUENCE)

    def _capture(self, size: int) -> _Bucket:
        dev = self.device
        slots = self._slots(size)
        ids = torch.zeros(size, dtype=torch.int64, device=dev)
        seqpos = torch.arange(size, dtype=torch.int64, device=dev) % PAD_SEQUENCE
        cu = torch.full((slots + 1,), size, dtype=torch.int32, device=dev)
        cu[0] = 0
        bounds = list(range(0, size, PAD_SEQUENCE)) + [size]
        cu[: len(bounds)] = torch.tensor(bounds, dtype=torch.int32, device=dev)
        # max_length = size bounds every position and sizes the rotary tables once for this bucket
        pack = Pack(input_ids=ids, seqpos=seqpos, cu=cu, cu_cpu=None, max_length=size,
                    markers=torch.zeros(1, dtype=torch.int64, device=dev),
                    marker_cu=torch.zeros(2, dtype=torch.int32, device=dev), max_markers=1)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            self.model.body(pack)  # warm-up: rotary tables and workspace exist before capture
        torch.cuda.current_stream(dev).wait_stream(stream)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self.pool):
            out = self.model.body(pack)
        keep = (self.model._workspace, *[t for pair in self.model._tables.values() for t in pair])
        return _Bucket(size, ids, seqpos, cu, pack, graph, out, keep)

    def bucket_for(self, p: Any) -> _Bucket | None:
        """The smallest bucket holding pack ``p``, or None when it runs the plain path."""
        if p.segment_ids_cpu is not None and bool((p.segment_ids_cpu != 0).any()):
            return None  # branched layouts plan their virtual sequences per pack
        if getattr(p, "pixel_values", None) is not None:
            return None  # images plan their rows per pack
        t = int(p.input_ids.numel())
        n = int(p.cu.numel()) - 1
        if n > self.max_sequences:
            return None
        for b in self.buckets:
            if b.size >= t:
                return b
        return None

    def __call__(self, p: Any) -> torch.Tensor:
        b = self.bucket_for(p)
        if b is None:
            return self.model(p)
        self.model.plan(p)  # the plain path's refusals of malformed packs (no plan: a covered pack has no branches)
        t = int(p.input_ids.numel())
        n = int(p.cu.numel()) - 1
        b.ids[:t].copy_(p.input_ids, non_blocking=True)
        b.seqpos[:t].copy_(p.seqpos, non_blocking=True)
        # boundaries: the pack's, then padding sequences over rows t .. size, then empty sequences
        pad = np.arange(t, b.size, PAD_SEQUENCE, dtype=np.int64)[1:] if b.size > t else np.zeros(0, dtype=np.int64)
        tail = np.concatenate([pad, [b.size]]) if b.size > t else np.zeros(0, dtype=np.int64)
        b.cu[: n + 1].copy_(p.cu, non_blocking=True)
        if len(tail):
            b.cu[n + 1: n + 1 + len(tail)].copy_(torch.from_numpy(tail.astype(np.int32)), non_blocking=True)
        b.cu[n + 1 + len(tail):].fill_(b.size)
        if b.size > t:  # padding rows: ids 0, positions restarting in every padding sequence
            b.ids[t:].zero_()
            b.seqpos[t:].copy_(torch.arange(b.size - t, device=self.device) % PAD_SEQUENCE, non_blocking=True)
        b.graph.replay()
        return self.model.head(b.out[:t], p)

    def release(self) -> None:
        """Drops the graphs (and the memory they hold)."""
        self.buckets.clear()
