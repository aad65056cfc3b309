"""The drop-in boundary on the GPU, as the reference's Decider binds it (decider.py:35-36, 117-118):

    self.model = family.Packed(ckpt.backbone, attention)   ->  Packed.from_backbone(ckpt.backbone, attention)
    self.readout = ckpt.readout                            ->  Readout.from_reference(ckpt.readout)
    hidden = self.model(pack(sequences, backbone, device)); flat = self.readout(hidden).cpu()

The backbone is the Transformers module the reference wraps (random-init weights of the golden cases, on the GPU in
bf16 as it is served; ``--fp8`` passed as ``fp8=True``), the head a module with the reference ``Readout``'s attributes,
and the pack an object with exactly the reference ``Pack``'s fields (model/packed.py:29-61: M-RoPE ``rope`` for joint
layouts, ``segments``, ``plan`` and the image fields left empty). The forward through these constructors must equal
``Packed(spec, weights)`` bit for bit and meet the golden bar against the reference's own outputs."""

import types

import numpy as np
import pytest
import torch

from backbones import to_dtype
from golden_cases import READOUT_BOUND, load, readout_bar
from karpo_decision_b200 import Packed, Readout, from_arrays
from test_dropin import DROPIN_CASES, backbone_of

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


class ReferenceReadout(torch.nn.Module):
    """The reference head's interface (model/readout.py:12-33): ``weight`` (codes, hidden) float32 and ``cap``."""

    def __init__(self, rows: np.ndarray, cap):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.from_numpy(rows).float())
        self.cap = cap


def reference_pack(arrays: dict, device) -> types.SimpleNamespace:
    """A pack with the reference ``Pack``'s field set, as its ``pack()`` fills them (model/packed.py:73-105)."""
    p = from_arrays(arrays, device)
    blocks = p.segment_ids is not None
    t = p.input_ids.numel()
    rope = None if blocks else p.seqpos.view(1, 1, t).expand(3, 1, t).contiguous()  # text: 0..n-1 on each axis
    return types.SimpleNamespace(
        input_ids=p.input_ids, seqpos=p.seqpos, cu=p.cu, cu_cpu=p.cu_cpu, max_length=p.max_length, markers=p.markers,
        marker_cu=p.marker_cu, max_markers=p.max_markers, segment_ids=p.segment_ids,
        segment_ids_cpu=p.segment_ids_cpu, rope=rope, pixel_values=None, image_grid_thw=None,
        image_position_ids=None, segments=1, plan=None)


@pytest.mark.parametrize("name", [*DROPIN_CASES, "qwen_tiny_fp8", "gemma_tiny_fp8", "gemma_blocks", "qwen_0p8b"])
def test_forward_through_the_drop_in_constructors(name):
    spec, weights, arrays, expected = load(name)
    fp8 = name.endswith("_fp8")
    backbone = backbone_of(spec, weights)
    lm = getattr(backbone, "language_model", backbone)
    to_dtype(lm.to(DEV), torch.bfloat16)  # the served backbone: on the GPU in bf16 (rotary frequencies in float32)
    model = Packed.from_backbone(backbone, spec.attention, fp8=fp8)
    head = Readout.from_reference(ReferenceReadout(weights["readout"], spec.logit_cap).to(DEV))
    assert model.spec.layers == spec.layers and model.device.type == "cuda"
    hidden = model(reference_pack(arrays, DEV))
    logits = head(hidden).cpu().numpy()
    direct = Packed(spec, weights, DEV, fp8=fp8)(from_arrays(arrays, DEV))
    assert torch.equal(hidden, direct)  # the same weights in the same layouts: the same bits
    if fp8:  # the tiny FP8 fixtures are the float32 FP8 forward, compared in test_gpu_packed.py
        return
    want = expected["logits"]
    bound = READOUT_BOUND
    if "logits_fp32" in expected:  # full width: the reference's own bf16 noise (test_gpu_wide.py)
        want = expected["logits_fp32"]
        bound = max(READOUT_BOUND, 1.25 * float(np.abs(expected["logits"] - want).max()))
    err, agree, ties = readout_bar(logits, want, bound)
    print(f"{name}: readout through from_backbone / from_reference, max-abs vs reference {err:.4f}, top answers "
          f"agree on {agree:.1%} ({ties} near ties)")
