"""Host planning of packs whose sequences are block layouts (Gemma 4 multi-question requests) and of packs with image
soft tokens: which rows each attention call reads, computed once per pack on the host and copied to the device
before any layer is queued.

The design works on a table of *blocks* rather than walking the pack sequence by sequence. A block is a maximal run
of rows of one sequence with one segment id. A sequence is valid when its blocks carry the ids 0, 1, 2, ... in order:
block 0 is the shared block (or the sequence's only block), blocks 1.. are branches whose positions continue after
the shared block. Every block is one *virtual sequence* of queries (its own rows). Its keys are at most two row spans,
held as (start, length) pairs for every block at once:

- a prefix span: nothing for block 0; for a branch, the shared block in global layers, and in sliding layers the
  shared block's last window - 1 rows (the window reaches back that far from the branch's first position);
- its own rows.

The key rows of all virtual sequences are then one vectorized expansion of those spans (``_expand``). This is the
same visibility as the reference's block plan (families/gemma/packed.py:54-151), whose integer results these must
equal; the tests check them against the oracle's restatement.

Images (families/gemma/vision.py:146-210) are planned the same way: each run of soft-token rows is one virtual
sequence of queries whose keys are a prefix span (the rows before it in its block that the sliding window reaches,
or, for an image in a branch, the part of the shared block the window reaches by position) and its own block's rows
up to the image's end.
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


def _expand(starts: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    """Concatenation of the ranges [starts[i], starts[i] + lengths[i]) in order, without a Python loop."""
    starts = np.asarray(starts, dtype=np.int64)
    lengths = np.asarray(lengths, dtype=np.int64)
    total = int(lengths.sum())
    if total == 0:
        return np.zeros(0, dtype=np.int64)
    ends = np.cumsum(lengths)
    # each output element's offset within its range, plus its range's start
    first = np.repeat(ends - lengths, lengths)
    return np.arange(total, dtype=np.int64) - first + np.repeat(starts, lengths)


def _bounds(lengths: np.ndarray) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(lengths, dtype=np.int64)])


def _spans(prefix_start, prefix_len, own_start, own_len) -> tuple[np.ndarray, np.ndarray]:
    """Key rows and their bounds for virtual sequences with keys = prefix span, then own span."""
    starts = np.stack([prefix_start, own_start], axis=1).reshape(-1)
    lengths = np.stack([prefix_len, own_len], axis=1).reshape(-1)
    return _expand(starts, lengths), _bounds(prefix_len + own_len)


@dataclass
class _Blocks:
    start: np.ndarray  # first row of each block
    length: np.ndarray
    label: np.ndarray  # its segment id
    seq_start: np.ndarray  # first row of its sequence
    shared_len: np.ndarray  # length of its sequence's block 0


def _blocks(cu: np.ndarray, segments: np.ndarray) -> _Blocks:
    """The pack's block table; ValueError when a sequence's segment ids are not 0, 1, 2, ... block by block."""
    cu = np.asarray(cu, dtype=np.int64)
    segments = np.asarray(segments).astype(np.int64, copy=False)
    t = len(segments)
    new = np.zeros(t, dtype=bool)
    if t:
        new[0] = True
        new[1:] = segments[1:] != segments[:-1]
    inner = cu[(cu > 0) & (cu < t)]
    new[inner] = True  # a sequence start always opens a block
    start = np.flatnonzero(new).astype(np.int64)
    length = np.diff(np.append(start, t))
    label = segments[start]
    seq = np.searchsorted(cu, start, side="right") - 1
    first_block = np.searchsorted(start, cu[:-1])  # index of each sequence's block 0
    rank = np.arange(len(start)) - first_block[seq]
    bad = np.flatnonzero(label != rank)
    if bad.size:
        s = int(seq[bad[0]])
        ids = label[first_block[s]:(first_block[s + 1] if s + 1 < len(first_block) else len(start))].tolist()
        raise ValueError(f"sequence {s} has segment ids {ids} block by block; a block layout is the shared block 0 "
                         f"followed by branches 1, 2, ...")
    shared_len = length[first_block][seq]
    return _Blocks(start=start, length=length, label=label, seq_start=cu[:-1][seq], shared_len=shared_len)


def marker_bounds(q_cu: list[int] | np.ndarray, markers: np.ndarray) -> list[int]:
    """Bounds of the (sorted) markers over virtual sequences ``q_cu``, refusing the layouts the reference refuses
    (families/gemma/packed.py:136-143): a block or branch reads out at most one marker, at its last row."""
    q_cu = np.asarray(q_cu, dtype=np.int64)
    markers = np.asarray(markers, dtype=np.int64)
    m_cu = np.searchsorted(markers, q_cu)
    count = np.diff(m_cu)
    last = q_cu[1:] - 1
    has = count == 1
    wrong = count > 1
    wrong[has] |= markers[m_cu[:-1][has]] != last[has]
    if wrong.any():
        v = int(np.flatnonzero(wrong)[0])
        raise ValueError(f"block {v} (rows {int(q_cu[v])}..{int(last[v])}) has {int(count[v])} readout markers; "
                         f"a block reads out at most one, at its last row")
    return m_cu.tolist()


def block_plan(cu_cpu: Any, segment_ids_cpu: Any, window: int, device: torch.device,
               markers_cpu: Any = None) -> BlockPlan:
    """The virtual sequences of a pack of block layouts. ``window`` is the sliding layers' (a row sees itself and
    window - 1 rows before it). Raises ValueError on malformed segment ids; with ``markers_cpu``, also plans the
    markers per virtual sequence and refuses misplaced ones."""
    cu = np.asarray(cu_cpu.numpy() if isinstance(cu_cpu, torch.Tensor) else cu_cpu, dtype=np.int64)
    seg = segment_ids_cpu.numpy() if isinstance(segment_ids_cpu, torch.Tensor) else np.asarray(segment_ids_cpu)
    b = _blocks(cu, seg)
    branch = b.label > 0
    zero = np.zeros_like(b.start)
    # global layers: a branch sees the whole shared block
    g_rows, g_cu = _spans(b.seq_start, np.where(branch, b.shared_len, zero), b.start, b.length)
    # sliding layers: the shared block's last window - 1 rows
    tail = np.minimum(b.shared_len, max(window - 1, 0))
    s_rows, s_cu = _spans(b.seq_start + b.shared_len - tail, np.where(branch, tail, zero), b.start, b.length)
    q_cu = _bounds(b.length)

    def dev(x, dtype):
        return torch.as_tensor(np.asarray(x), dtype=dtype).to(device, non_blocking=False)

    m_cu = None if markers_cpu is None else dev(marker_bounds(q_cu, np.asarray(markers_cpu)), torch.int32)
    return BlockPlan(q_cu=dev(q_cu, torch.int32), g_rows=dev(g_rows, torch.int64), g_cu=dev(g_cu, torch.int32),
                     s_rows=dev(s_rows, torch.int64), s_cu=dev(s_cu, torch.int32), max_q=int(b.length.max()),
                     m_cu=m_cu)


@dataclass
class ImagePlan:
    """Each image's soft-token rows in a pack, for the sliding layers (families/gemma/vision.py:146-210): every soft
    token's row (images in pack order, each a run of rows), and per image the key rows it sees, whose positions run
    contiguously up to the image's end (the window before the image inside what its block reads, then the image
    itself), so the end-aligned window (W - 1, unbounded right) of the varlen contract over those keys is the
    reference's mask: a key at or after the query's position - (W - 1), the whole image included."""

    rows: torch.Tensor  # int64 soft-token rows, image by image
    q_cu: torch.Tensor  # (images + 1,) int32 bounds over ``rows``
    keys: torch.Tensor  # int64 key rows, image by image
    k_cu: torch.Tensor  # (images + 1,) int32 bounds over ``keys``
    max_q: int


def image_plan(input_ids: np.ndarray, bounds: list[int], segments: np.ndarray | None, positions: np.ndarray,
               soft: int, window: int, device: torch.device) -> ImagePlan:
    """The plan of a pack's images from host arrays (``soft``: the soft-token id). Refuses, as the reference does, a
    pack with images but no soft token and an image longer than the sliding window. An image in a shared block (or a
    sequence's only block) sees its block's rows within the window before it; an image in a branch sees the part of
    the shared block the window reaches by position, then its branch's rows before it; both see their whole self."""
    input_ids = np.asarray(input_ids)
    positions = np.asarray(positions, dtype=np.int64)
    segments = np.zeros(len(input_ids), dtype=np.int64) if segments is None else np.asarray(segments)
    rows = np.flatnonzero(input_ids == soft).astype(np.int64)
    if rows.size == 0:
        raise ValueError("a pack with images has no image soft tokens")
    opens = np.flatnonzero(np.diff(rows, prepend=rows[0] - 2) != 1)  # the first soft token of each image
    s = rows[opens]
    e = np.append(rows[opens[1:] - 1], rows[-1]) + 1
    size = e - s
    if (size > window).any():
        i = int(np.argmax(size > window))
        raise ValueError(f"image {i} has {int(size[i])} soft tokens, more than the sliding window ({window})")
    b = _blocks(np.asarray(bounds, dtype=np.int64), segments)
    blk = np.searchsorted(b.start, s, side="right") - 1  # the block holding each image
    in_branch = b.label[blk] > 0
    reach = max(window - 1, 0)
    shared = b.shared_len[blk]
    seq0 = b.seq_start[blk]
    # image in block 0: one span, the rows from max(block start, s - reach) to the image's end
    own_start = np.where(in_branch, b.start[blk], np.maximum(b.start[blk], s - reach))
    # image in a branch: the shared positions from max(0, position(s) - reach) on (its position counts from the
    # shared block's start), capped at the shared block's end, then the branch's rows up to the image's end
    first = np.minimum(np.maximum(0, positions[s] - reach), shared)
    prefix_start = np.where(in_branch, seq0 + first, 0)
    prefix_len = np.where(in_branch, shared - first, 0)
    keys, k_cu = _spans(prefix_start, prefix_len, own_start, e - own_start)

    def dev(x, dtype):
        return torch.as_tensor(np.asarray(x), dtype=dtype).to(device)

    return ImagePlan(rows=dev(rows, torch.int64), q_cu=dev(_bounds(size), torch.int32), keys=dev(keys, torch.int64),
                     k_cu=dev(k_cu, torch.int32), max_q=int(size.max()))
