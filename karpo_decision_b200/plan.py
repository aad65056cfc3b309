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


@dataclass
class ImagePlan:
    """Each image's soft-token rows in a pack of block layouts, for the sliding layers (families/gemma/vision.py:
    146-210): every soft token's row (images in pack order, each a run of rows), and per image the key rows it sees,
    whose positions run contiguously up to the image's end (the window before the image inside what its block reads,
    then the image itself), so the end-aligned window (W - 1, unbounded right) of the varlen contract over those keys
    is the reference's mask: a key at or after the query's position - (W - 1), the whole image included."""

    rows: torch.Tensor  # int64 soft-token rows, image by image
    q_cu: torch.Tensor  # (images + 1,) int32 bounds over ``rows``
    keys: torch.Tensor  # int64 key rows, image by image
    k_cu: torch.Tensor  # (images + 1,) int32 bounds over ``keys``
    max_q: int


def image_plan(input_ids: np.ndarray, bounds: list[int], segments: np.ndarray | None, positions: np.ndarray,
               soft: int, window: int, device: torch.device) -> ImagePlan:
    """The plan of a pack's images from host arrays (``soft``: the soft-token id), with the reference's refusals:
    no soft token in a pack with images, an image longer than the sliding window (families/gemma/vision.py:174-196).
    An image in a shared block (or a sequence's only block) sees the rows before it within the window; one in a branch
    sees the shared block's rows within the window by position and its branch's rows before it."""
    input_ids = np.asarray(input_ids)
    positions = np.asarray(positions, dtype=np.int64)
    segments = np.zeros(len(input_ids), dtype=np.int64) if segments is None else np.asarray(segments)
    rows = np.flatnonzero(input_ids == soft)
    if rows.size == 0:
        raise ValueError("a pack with images has no image soft tokens")
    breaks = (np.flatnonzero(rows[1:] != rows[:-1] + 1) + 1).tolist()
    q_cu, k_cu, keys = [0], [0], []
    max_q = 0
    for a, b in zip([0, *breaks], [*breaks, len(rows)], strict=True):
        s, e = int(rows[a]), int(rows[b - 1]) + 1
        if e - s > window:
            raise ValueError(f"an image of {e - s} soft tokens is longer than the sliding window ({window})")
        start = bounds[int(np.searchsorted(bounds, s, side="right")) - 1]
        if int(segments[s]) == 0:
            seen = np.arange(max(start, s - (window - 1)), e)
        else:
            shared = int((segments[start:s] == 0).sum())  # the shared block's length: branch positions follow it
            branch = s - (int(positions[s]) - shared)  # the branch's first row
            first = min(max(0, int(positions[s]) - (window - 1)), shared)  # the first shared position it sees
            seen = np.concatenate([np.arange(start + first, start + shared), np.arange(branch, e)])
        keys.append(seen)
        q_cu.append(q_cu[-1] + e - s)
        k_cu.append(k_cu[-1] + len(seen))
        max_q = max(max_q, e - s)

    def dev(x, dtype):
        return torch.as_tensor(np.asarray(x), dtype=dtype).to(device)

    return ImagePlan(rows=dev(rows, torch.int64), q_cu=dev(q_cu, torch.int32),
                     keys=dev(np.concatenate(keys), torch.int64), k_cu=dev(k_cu, torch.int32), max_q=max_q)
