"""The boundary object: sequences laid end to end into one padding-free pack, as the reference's ``Pack`` / ``pack``
(model/packed.py:29-105) define it for text-only sequences. The packed forward (``Packed``) reads the same attributes
from the reference's own ``Pack``, so either can be passed in.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch


@dataclass
class Pack:
    """Sequences laid end to end, on the model's device (model/packed.py:29-61)."""

    input_ids: torch.Tensor  # (T,) int64
    seqpos: torch.Tensor  # (T,) int64 position inside the token's own sequence (block layouts: the layout's)
    cu: torch.Tensor  # (n + 1,) int32 sequence boundaries
    cu_cpu: torch.Tensor | None  # the same, int64 on CPU
    max_length: int
    markers: torch.Tensor  # (M,) int64 rows of the readout markers, in pack order
    marker_cu: torch.Tensor  # (n + 1,) int32 marker boundaries per sequence
    max_markers: int
    segment_ids: torch.Tensor | None = None  # block layouts: 0 a sequence's shared block, k its k-th branch
    segment_ids_cpu: torch.Tensor | None = None
    rope: torch.Tensor | None = None  # Qwen joint layouts with images: (3, 1, T) M-RoPE positions
    plan: Any = None
    markers_cpu: torch.Tensor | None = None  # the markers on the host (planning checks need no device read)
    pixel_values: torch.Tensor | None = None  # images: what the model's image_features reads (model/packed.py:43-48)
    image_position_ids: torch.Tensor | None = None
    image_grid_thw: torch.Tensor | None = None  # Qwen joint layouts: each image's (t, h, w) grid of patches

    @property
    def tokens(self) -> int:
        return int(self.input_ids.numel())


def pack(sequences: Sequence[Any], device: torch.device, blocks: bool = False) -> Pack:
    """Packs sequences (objects with ``input_ids`` and ``markers`` 1-D tensors, and for block layouts ``positions``
    and ``segment_ids``) as model/packed.py:73-105 does for text: ids and positions concatenated, int32 boundaries,
    markers shifted to global rows; copies are non-blocking from host memory."""
    lengths = [int(s.input_ids.numel()) for s in sequences]
    if not lengths:
        raise ValueError("a pack needs at least one sequence")
    cu_cpu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int64)
    starts = cu_cpu[:-1].tolist()
    if blocks:
        seqpos = torch.cat([s.positions for s in sequences])
        segment_ids = torch.cat([s.segment_ids for s in sequences]).to(torch.int32)
    else:
        seqpos = torch.cat([torch.arange(n) for n in lengths])
        segment_ids = None
    counts = [int(s.markers.numel()) for s in sequences]
    markers = torch.cat([s.markers + start for s, start in zip(sequences, starts, strict=True)])
    return Pack(
        input_ids=torch.cat([s.input_ids for s in sequences]).to(device, non_blocking=True),
        seqpos=seqpos.to(device, torch.int64, non_blocking=True),
        cu=cu_cpu.to(device, torch.int32, non_blocking=True),
        cu_cpu=cu_cpu,
        max_length=max(lengths),
        markers=markers.to(device, torch.int64, non_blocking=True),
        marker_cu=torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32).to(device),
        max_markers=max(counts),
        segment_ids=None if segment_ids is None else segment_ids.to(device, non_blocking=True),
        segment_ids_cpu=segment_ids,
        markers_cpu=markers.to(torch.int64),
    )


def from_arrays(arrays: dict[str, np.ndarray], device: torch.device, pinned: bool = False) -> Pack:
    """A pack from host arrays (``synthetic.synthetic_pack_arrays`` layout: input_ids, seqpos, cu, markers,
    marker_cu, and segment_ids for block layouts; with images, pixel_values and, for Qwen joint layouts, the (3, T)
    M-RoPE positions ``rope``); ``pinned`` stages them in page-locked memory so the copies are asynchronous."""

    def host(a, dtype):
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dtype)
        return t.pin_memory() if pinned else t

    cu = arrays["cu"]
    lengths = np.diff(cu)
    counts = np.diff(arrays["marker_cu"])
    segments = arrays.get("segment_ids")
    seg_cpu = None if segments is None else torch.from_numpy(np.asarray(segments, dtype=np.int32))
    return Pack(
        input_ids=host(arrays["input_ids"], torch.int64).to(device, non_blocking=True),
        seqpos=host(arrays["seqpos"], torch.int64).to(device, non_blocking=True),
        cu=host(cu, torch.int32).to(device, non_blocking=True),
        cu_cpu=torch.from_numpy(np.asarray(cu, dtype=np.int64)),
        max_length=int(lengths.max()),
        markers=host(arrays["markers"], torch.int64).to(device, non_blocking=True),
        marker_cu=host(arrays["marker_cu"], torch.int32).to(device, non_blocking=True),
        max_markers=int(counts.max()),
        segment_ids=None if seg_cpu is None else seg_cpu.to(device, non_blocking=True),
        segment_ids_cpu=seg_cpu,
        markers_cpu=torch.from_numpy(np.asarray(arrays["markers"], dtype=np.int64)),
        pixel_values=(torch.from_numpy(np.ascontiguousarray(arrays["pixel_values"])).to(device)
                      if arrays.get("pixel_values") is not None else None),
        rope=(host(arrays["rope"], torch.int64).reshape(len(arrays["rope"]), 1, -1).to(device, non_blocking=True)
              if arrays.get("rope") is not None else None),
    )
