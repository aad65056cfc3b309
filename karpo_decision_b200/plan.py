"""The virtual sequences of a pack of block layouts (the reference's families/gemma/packed.py:54-151, ``BlockPlan``
and ``block_plan``), computed once per pack on the host from ``cu_cpu`` and ``segment_ids_cpu`` and copied to the
device before any layer is queued.

A sequence of one block attends within itself. A branched sequence (segment 0 the shared block, then branches 1, 2,
...) becomes virtual sequences: the shared block attending to itself, then each branch attending to the shared block
and itself: global layers see the whole shared block, sliding layers its last window - 1 rows (a branch's positions
continue after the shared block, so the window reaches that far). Keys are gathered per virtual sequence in that
order; attention aligns each virtual sequence's queries with the end of its keys.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch


@dataclass
class BlockPlan:
    q_cu: torch.Tensor  # (v + 1,) int32 query bounds of the virtual sequences over the pack's rows
    g_rows: torch.Tensor  # int64 key rows of global layers, virtual sequence by virtual sequence
    g_cu: torch.Tensor  # (v + 1,) int32 bounds over g_rows
    s_rows: torch.Tensor  # int64 key rows of sliding layers
    s_cu: torch.Tensor  # (v + 1,) int32 bounds over s_rows
    max_q: int
    m_cu: torch.Tensor | None = None  # (v + 1,) int32 marker bounds over the virtual sequences (markers in pack order)


def marker_bounds(q_cu: list[int], markers: np.ndarray) -> list[int]:
    """The markers' bounds over virtual sequences ``q_cu`` (pack rows), refusing what the reference refuses: a block's
    readout marker is its last token, at most one per block or branch (families/gemma/packed.py:136-143)."""
    markers = np.asarray(markers, dtype=np.int64)
    m_cu = np.searchsorted(markers, np.asarray(q_cu, dtype=np.int64)).tolist()
    for qb, ma, mb in zip(q_cu[1:], m_cu[:-1], m_cu[1:], strict=True):
        if mb - ma > 1 or (mb > ma and int(markers[ma]) != qb - 1):
            raise ValueError("a block's readout marker must be its last token, one per branch")
    return m_cu


def block_plan(cu_cpu: torch.Tensor, segment_ids_cpu: torch.Tensor, window: int, device: torch.device,
               markers_cpu: Any = None) -> BlockPlan:
    """Raises ValueError on segments that are not a shared block followed by branches 1, 2, ... (the reference's
    refusal, families/gemma/packed.py:116-118); with ``markers_cpu``, also plans (and checks) the markers per virtual
    sequence."""
    bounds = cu_cpu.tolist()
    segments = segment_ids_cpu.numpy() if isinstance(segment_ids_cpu, torch.Tensor) else np.asarray(segment_ids_cpu)
    q_cu, g_cu, s_cu = [0], [0], [0]
    g_rows: list[np.ndarray] = []
    s_rows: list[np.ndarray] = []
    for a, b in zip(bounds[:-1], bounds[1:], strict=True):
        seg = segments[a:b]
        change = (np.flatnonzero(seg[1:] != seg[:-1]) + 1).tolist()
        starts, ends = [0, *change], [*change, b - a]
        labels = [int(seg[i]) for i in starts]
        if labels != list(range(len(labels))):
            raise ValueError(f"segments {labels} are not a shared block followed by branches 1, 2, ...")
        shared = ends[0]
        own = np.arange(a, a + shared, dtype=np.int64)
        tail = own[max(0, shared - (window - 1)):]
        q_cu.append(a + shared)
        g_rows.append(own)
        s_rows.append(own)
        g_cu.append(g_cu[-1] + shared)
        s_cu.append(s_cu[-1] + shared)
        for start, end in zip(starts[1:], ends[1:], strict=True):
            rows = np.arange(a + start, a + end, dtype=np.int64)
            q_cu.append(a + end)
            g_rows.append(np.concatenate([own, rows]))
            s_rows.append(np.concatenate([tail, rows]))
            g_cu.append(g_cu[-1] + shared + len(rows))
            s_cu.append(s_cu[-1] + len(tail) + len(rows))

    def dev(x, dtype):
        return torch.as_tensor(np.asarray(x), dtype=dtype).to(device, non_blocking=False)

    m_cu = None if markers_cpu is None else dev(marker_bounds(q_cu, np.asarray(markers_cpu)), torch.int32)
    return BlockPlan(q_cu=dev(q_cu, torch.int32), g_rows=dev(np.concatenate(g_rows), torch.int64),
                     g_cu=dev(g_cu, torch.int32), s_rows=dev(np.concatenate(s_rows), torch.int64),
                     s_cu=dev(s_cu, torch.int32), max_q=int(np.diff(q_cu).max()), m_cu=m_cu)
