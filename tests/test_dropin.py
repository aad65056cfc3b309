"""The drop-in constructors on the host: ``Packed.from_backbone`` over the Transformers modules the reference wraps
(decider.py:35, ``ckpt.family.Packed(ckpt.backbone, attention)``) infers the same shape and lays out the same weights
as ``Packed(spec, weights)``; ``Readout.from_reference`` reads the reference ``Readout``'s rows and cap
(decider.py:36). Runs on the CPU (no kernel is launched); the GPU forward through them is in test_gpu_dropin.py."""

import types

import pytest
import torch

from backbones import gemma_lm, qwen_backbone
from golden_cases import load
from karpo_decision_b200.packed import Packed, Projection

CPU = torch.device("cpu")
#: plain Qwen, partial rotary, the hybrid stack with Gated DeltaNet layers, Gemma's sliding/global layers,
#: Gemma 4's head-512 global layers with shared keys and values and proportional RoPE, and bidirectional checkpoints
DROPIN_CASES = ["qwen_tiny", "qwen_partial", "qwen_hybrid", "gemma_tiny", "gemma_global512", "qwen_bidir",
                "gemma_bidir"]


def backbone_of(spec, weights):
    """The module the reference's Decider holds as ``ckpt.backbone`` for this shape (Gemma: the multimodal model's
    ``language_model`` and ``config``, no vision tower)."""
    if spec.family == "qwen":
        return qwen_backbone(spec, weights)
    return types.SimpleNamespace(language_model=gemma_lm(spec, weights), config=types.SimpleNamespace(image_token_id=None))


def _tensors(model: Packed):
    """Every weight tensor the model holds, in a fixed order."""
    out = [model.embed_tokens, model.norm]
    for layer in model.layers:
        for value in vars(layer).values():
            items = value if isinstance(value, list) else [value]
            for item in items:
                if isinstance(item, tuple):
                    item = item[0]
                if isinstance(item, Projection):
                    out += [item.weight] + ([item.scale] if item.scale is not None else [])
                elif isinstance(item, torch.Tensor):
                    out.append(item)
        if layer.mixer is not None:
            out += [p.weight for p, _, _ in layer.mixer.proj]
            out += [layer.mixer.conv, layer.mixer.a_log, layer.mixer.dt_bias, layer.mixer.norm]
    return out


@pytest.mark.parametrize("name", DROPIN_CASES)
def test_from_backbone_infers_the_shape_and_lays_out_the_same_weights(name):
    spec, weights, _, _ = load(name)
    model = Packed.from_backbone(backbone_of(spec, weights), spec.attention, device=CPU)
    direct = Packed(spec, weights, CPU)
    for field in ("family", "layers", "hidden", "heads", "kv_heads", "head_dim", "intermediate", "vocab", "eps",
                  "partial_rotary", "attention", "full_every", "k_eq_v", "global_rope"):
        assert getattr(model.spec, field) == getattr(spec, field), field
    if spec.family == "gemma":
        for field in ("window", "rope_theta", "rope_theta_local", "logit_cap", "global_partial_rotary"):
            assert getattr(model.spec, field) == getattr(spec, field), field
        assert (model.spec.global_head_dim or spec.head_dim) == (spec.global_head_dim or spec.head_dim)
    assert model.types == direct.types and model.prune_last == direct.prune_last
    a, b = _tensors(model), _tensors(direct)
    assert len(a) == len(b)
    for x, y in zip(a, b, strict=True):
        assert x.shape == y.shape and torch.equal(x, y)
    for kind in model._inv_freq:
        assert torch.equal(model._inv_freq[kind], direct._inv_freq[kind])


def test_readout_from_reference_reads_rows_and_cap():
    from karpo_decision_b200.packed import Readout

    class ReferenceReadout(torch.nn.Module):  # model/readout.py:12-33: weight (codes, hidden) float32, cap
        def __init__(self, rows, cap):
            super().__init__()
            self.weight = torch.nn.Parameter(rows.float())
            self.cap = cap

    rows = torch.randn(5, 64)
    head = Readout.from_reference(ReferenceReadout(rows, 30.0), device=CPU)
    assert torch.equal(head.weight.cpu(), rows) and head.cap == 30.0


def test_from_backbone_reads_the_mrope_sections_and_image_token():
    """A Qwen3.5 backbone's interleaved M-RoPE sections and image token reach the spec and the model, and its vision
    tower is wired as the image-feature source (families/qwen/packed.py:70, :161-163)."""
    spec, weights, _, _ = load("qwen_images")
    model = Packed.from_backbone(qwen_backbone(spec, weights), device=CPU)
    assert model.spec.mrope_section == (12, 10, 10)
    assert model.image_token_id == spec.vocab - 1 and model.image_features is not None
    axes = model.spec.pair_axes()
    assert axes[:7] == [0, 1, 2, 0, 1, 2, 0] and axes[30:] == [0, 0] and len(axes) == 32
