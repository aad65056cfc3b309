"""Generates the golden fixtures of this directory by running the reference implementation itself.

Run in a container where the karpo-decision source tree is available (``--reference`` points at its root; the
fixtures are committed, so the GPU box never needs it):

    python tests/golden/make_golden.py --reference <karpo-decision checkout>

For each case it builds a random-init Transformers backbone (Qwen3_5Model with full-attention layers, or
Gemma4TextModel with 5 sliding : 1 global layers) with the seeded weights of ``karpo_decision_b200.synthetic``,
packs seeded sequences with the reference's own ``pack`` and runs the reference's own ``families.*.Packed`` and
``Readout`` on CPU in float32. FP8 cases run the reference's own ``serve.qwen_fp8.quantize`` / ``serve.fp8.quantize``.

Harness-only substitutions (the CPU has none of the reference's GPU kernels), each a restatement of the contract the
reference's own tests use:
- varlen attention: ``varlen_contract`` below, the end-aligned window contract of the reference's
  tests/test_gemma_blocks.py:28-43, replaces torch's ``varlen_attn`` / FA4;
- ``torch._scaled_mm`` (rowwise scales are not implemented on CPU): ``(a.float() @ b.float()) * scale_a * scale_b``
  rounded to the output dtype, the documented semantics of rowwise scaling;
- Transformers 5.5 names a layer's kind ``layer_type``; the reference reads ``block_type``: aliased per layer;
- ``transformers.models.gemma4_unified`` (newer Transformers) is absent: stubbed, it is only imported for a type;
- flash-linear-attention's GPU kernels for the Gated DeltaNet: ``delta_rule_contract`` (Transformers' recurrent
  torch implementation per packed sequence) and ``conv_contract`` (the causal convolution cut at sequence starts).
"""

from __future__ import annotations

import argparse
import contextlib
import dataclasses
import hashlib
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

sys.path.insert(0, str(HERE.parent))
from backbones import gemma_lm, qwen_backbone, to_dtype, to_torch  # noqa: E402

from karpo_decision_b200.synthetic import (  # noqa: E402
    CONFIGS, Spec, numpy_weights, small, synthetic_block_arrays, synthetic_lengths, synthetic_pack_arrays)


#: The image soft-token id of the image cases (the last vocabulary id; other tokens never take it).
IMAGE_TOKEN = 4095


def oracle_bf16(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to bf16 (round to nearest even), kept as float32."""
    return torch.from_numpy(x).bfloat16().float().numpy()


def varlen_contract(q, k, v, cu_q, cu_k, max_q, max_k, scale=None, window_size=(-1, -1), enable_gqa=False):
    """Per sequence, query i sees key j when i + (Lk - Lq) - left <= j <= i + (Lk - Lq) + right (-1 unbounded)."""
    left, right = window_size
    outs = []
    for qa, qb, ka, kb in zip(cu_q[:-1].tolist(), cu_q[1:].tolist(), cu_k[:-1].tolist(), cu_k[1:].tolist(),
                              strict=True):
        if qb == qa:
            continue
        i = torch.arange(qb - qa)[:, None] + (kb - ka) - (qb - qa)
        j = torch.arange(kb - ka)[None, :]
        mask = torch.ones(qb - qa, kb - ka, dtype=torch.bool)
        if right >= 0:
            mask &= j <= i + right
        if left >= 0:
            mask &= j >= i - left
        outs.append(F.scaled_dot_product_attention(q[qa:qb].transpose(0, 1)[None], k[ka:kb].transpose(0, 1)[None],
                                                   v[ka:kb].transpose(0, 1)[None], attn_mask=mask, scale=scale,
                                                   enable_gqa=k.shape[1] != q.shape[1])[0].transpose(0, 1))
    return torch.cat(outs)


def delta_rule_contract(q, k, v, g, beta, initial_state=None, output_final_state=False,
                        use_qk_l2norm_in_kernel=False, cu_seqlens=None, cu_seqlens_cpu=None, **_):
    """flash-linear-attention's chunk_gated_delta_rule over packed sequences (its cu_seqlens contract: the state
    restarts from zero at every boundary), by Transformers' own recurrent torch implementation per sequence."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_recurrent_gated_delta_rule

    bounds = cu_seqlens_cpu.tolist() if cu_seqlens_cpu is not None else [0, q.shape[1]]
    outs = []
    for a, b in zip(bounds[:-1], bounds[1:], strict=True):
        o, _ = torch_recurrent_gated_delta_rule(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b], None, False,
                                                use_qk_l2norm_in_kernel)
        outs.append(o)
    return torch.cat(outs, 1), None


def conv_contract(x, weight, activation=None, cu_seqlens=None, cu_seqlens_cpu=None, **_):
    """flash-linear-attention's causal_conv1d over packed sequences: x (1, T, C), depthwise taps (C, K), no tap
    reaching before its sequence's start, float32 sums, the activation in float32, cast back to x's dtype."""
    bounds = cu_seqlens_cpu.tolist() if cu_seqlens_cpu is not None else [0, x.shape[1]]
    taps = weight.shape[1]
    xf, wf = x[0].float(), weight.float()
    out = torch.zeros_like(xf)
    for a, b in zip(bounds[:-1], bounds[1:], strict=True):
        for shift in range(taps):
            if b - a > shift:
                out[a + shift:b] += xf[a:b - shift] * wf[:, taps - 1 - shift]
    if activation in ("silu", "swish"):
        out = F.silu(out)
    return out.to(x.dtype)[None], None


def scaled_mm_contract(a, b, scale_a, scale_b, out_dtype=torch.bfloat16, **_):
    return ((a.float() @ b.float()) * scale_a * scale_b).to(out_dtype)


def import_reference(root: Path) -> None:
    sys.path.insert(0, str(root / "src"))
    if "transformers.models.gemma4_unified" not in sys.modules:
        pkg = types.ModuleType("transformers.models.gemma4_unified")
        mod = types.ModuleType("transformers.models.gemma4_unified.modeling_gemma4_unified")
        mod.Gemma4UnifiedModel = type("Gemma4UnifiedModel", (), {})
        pkg.modeling_gemma4_unified = mod
        sys.modules[pkg.__name__] = pkg
        sys.modules[mod.__name__] = mod
    with contextlib.suppress(ImportError):
        import pybase64  # noqa: F401
    if "pybase64" not in sys.modules:
        import base64
        stub = types.ModuleType("pybase64")
        stub.b64decode = lambda s, validate=False: base64.b64decode(s, validate=validate)
        sys.modules["pybase64"] = stub


def encoded(arrays: dict[str, np.ndarray], blocks: bool):
    from karpo_decision.encoding import Encoded

    out = []
    cu, markers, mcu = arrays["cu"], arrays["markers"], arrays["marker_cu"]
    for s in range(len(cu) - 1):
        a, b = int(cu[s]), int(cu[s + 1])
        local = torch.from_numpy(markers[mcu[s]:mcu[s + 1]] - a)
        n = b - a
        kw = {}
        if blocks and "segment_ids" in arrays:  # block layouts with branches (synthetic_block_arrays)
            kw = dict(positions=torch.from_numpy(arrays["seqpos"][a:b].copy()),
                      segment_ids=torch.from_numpy(arrays["segment_ids"][a:b].astype(np.int16)))
        elif blocks:
            kw = dict(positions=torch.arange(n), segment_ids=torch.zeros(n, dtype=torch.int16))
        if "image_grids" in arrays:  # Qwen joint layouts: this sequence's images, in row order
            grids = [g for row, g in zip(arrays["image_rows"], arrays["image_grids"]) if a <= row < b]
            if grids:
                ids = torch.from_numpy(arrays["input_ids"][a:b].copy())
                kw = dict(mm_token_type_ids=(ids == IMAGE_TOKEN).to(torch.int32), pixel_values=torch.zeros(1, 1),
                          image_grid_thw=torch.tensor(np.asarray(grids, dtype=np.int64)))
        out.append(Encoded(keys=tuple(f"q{i}" for i in range(len(local))), counts=(3,) * len(local),
                           input_ids=torch.from_numpy(arrays["input_ids"][a:b].copy()), markers=local, **kw))
    return out


def weights_digest(weights: dict[str, np.ndarray]) -> str:
    h = hashlib.sha256()
    for key in sorted(weights):
        h.update(key.encode())
        h.update(np.ascontiguousarray(weights[key], dtype=np.float32).tobytes())
    return h.hexdigest()


CASES = {
    # 2 layers, hidden 256, 4/2 heads of 64, SwiGLU 1024, vocab 4096; 8 sequences U[32, 512].
    "qwen_tiny": dict(spec=CONFIGS["tiny"], lengths=("uniform", 8, 32, 512), markers=(1, 1), fp8=False),
    # Partial rotary (Qwen3.5's real layers rotate a quarter of each head), 1-4 markers per sequence.
    "qwen_partial": dict(spec=small(CONFIGS["tiny"], partial_rotary=0.5, layers=2), lengths=("uniform", 6, 8, 200),
                         markers=(1, 4), fp8=False),
    # Gemma-shaped: 6 layers (5 sliding : 1 global), window 16, head 64.
    "gemma_tiny": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0),
                       lengths=("uniform", 6, 8, 96), markers=(1, 1), fp8=False),
    # FP8 projections (serve/qwen_fp8.py and serve/fp8.py).
    "qwen_tiny_fp8": dict(spec=CONFIGS["tiny"], lengths=("uniform", 4, 32, 160), markers=(1, 2), fp8=True),
    # Branched block layouts (blocks.py:194-214): shared blocks one short of, at and past the window, branches longer
    # than the window, single-block sequences beside branched ones (the reference's tests/test_gemma_blocks.py PACKS).
    "gemma_blocks": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0),
                         blocks=[(23, []), (21, [5, 7, 3]), (14, [4, 9]), (15, [3]), (16, [6, 2]),
                                 (17, [10, 1, 4]), (3, [20, 25])], fp8=False),
    "gemma_tiny_fp8": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0),
                           lengths=("uniform", 4, 8, 96), markers=(1, 1), fp8=True),
    # Bidirectional checkpoints (config.attention = "bidirectional"): full/global layers see their whole (virtual)
    # sequence and the last layer runs at the markers only (families/qwen/packed.py:127-140,
    # families/gemma/packed.py:267-281).
    "qwen_bidir": dict(spec=small(CONFIGS["tiny"], partial_rotary=0.5, attention="bidirectional"),
                       lengths=("uniform", 6, 8, 200), markers=(1, 4), fp8=False),
    "gemma_bidir": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0,
                                  attention="bidirectional"),
                        lengths=("uniform", 6, 8, 96), markers=(1, 1), fp8=False),
    # Gemma 4's real global layers: head 512, keys = values (attention_k_eq_v, one key/value head), proportional
    # RoPE over a quarter of the frequency pairs (families/gemma/global_attention.py, packed.py:183-193).
    "gemma_global512": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0,
                                      global_head_dim=512, global_kv_heads=1, k_eq_v=True, global_rope="proportional"),
                            lengths=("uniform", 5, 8, 160), markers=(1, 1), fp8=False),
    # Qwen3.5's hybrid stack: Gated DeltaNet layers with a full-attention layer every 2nd (the real 3:1 is
    # full_attention_interval 4), value heads twice the key heads.
    "qwen_hybrid": dict(spec=small(CONFIGS["tiny"], layers=4, full_every=2, partial_rotary=0.5, lin_k_heads=2,
                                   lin_v_heads=4, lin_k_dim=64, lin_v_dim=64),
                        lengths=("uniform", 6, 8, 200), markers=(1, 3), fp8=False),
    # Qwen3.5's real Gated DeltaNet head shape (128-dim keys and values, value heads twice the key heads), with
    # sequences shorter than, at, one past and several times the 128-token chunk of the tensor-core delta rule.
    "qwen_hybrid128": dict(spec=small(CONFIGS["tiny"], layers=4, full_every=2, partial_rotary=0.5, lin_k_heads=2,
                                      lin_v_heads=4, lin_k_dim=128, lin_v_dim=128),
                           lengths=("list", 100, 128, 129, 300, 517), markers=(1, 3), fp8=False),
    # Gemma 4 images (bidirectional checkpoints): soft-token runs in a single block, a shared block, a branch and at a
    # sequence's start; features stand in for the vision encoder's output (families/gemma/vision.py:136-144).
    "gemma_images": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0,
                                   attention="bidirectional"),
                         blocks=[(40, []), (30, [12, 20]), (25, [])], fp8=False,
                         images=[(10, 13), (45, 10), (85, 12), (102, 9)]),
    "gemma_blocks_bidir": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0,
                                         attention="bidirectional"),
                               blocks=[(23, []), (21, [5, 7, 3]), (14, [4, 9]), (3, [20, 25])], fp8=False),
}

#: BASELINE configurations 2-5 at full width, depth cut (a layer's arithmetic depends only on its kind, so a few
#: layers of each kind cover the whole stack), run through the reference's own bf16 path (the backbone cast to bf16,
#: as it is served) with ``dtype="bf16"``; the float32 run of the same case is stored beside it as the noise
#: reference. Gemma's vocabulary is cut to 8,192 rows (the configurations do not fix it).
WIDE = {
    # config 2: 0.8B Qwen-shaped, 2 layers, ~4k tokens of the [128, 8192] log-uniform mix, 1-4 markers
    "qwen_0p8b": dict(spec=small(CONFIGS["qwen-0.8b"], layers=2), lengths=("log", 4096, 128, 8192),
                      markers=(1, 4), fp8=False, dtype="bf16"),
    # config 3: 4B Qwen-shaped with FP8 projections, 2 layers, ~3k tokens of the [256, 16384] mix
    "qwen_4b_fp8": dict(spec=small(CONFIGS["qwen-4b"], layers=2), lengths=("log", 3072, 256, 16384, 2),
                        markers=(1, 4), fp8=True, dtype="bf16"),
    # config 4: 12B Gemma-shaped, head 256, window 1024, 5 sliding + 1 global layer; sequences one short of, at and
    # one past the window, and longer ones (the reference's window cases, tests/test_gemma_blocks.py:108-112)
    "gemma_12b": dict(spec=small(CONFIGS["gemma-12b"], layers=6, vocab=8192),
                      lengths=("list", 700, 1023, 1024, 1025, 3000), markers=(1, 1), fp8=False, dtype="bf16"),
    "gemma_12b_fp8": dict(spec=small(CONFIGS["gemma-12b"], layers=6, vocab=8192),
                          lengths=("list", 1023, 1025, 2048), markers=(1, 1), fp8=True, dtype="bf16"),
    # config 5: 31B Gemma-shaped with FP8 projections, 6 layers; multi-question requests as a shared block and
    # branches (shared blocks longer than the window), beside single-block ones
    "gemma_31b_fp8": dict(spec=small(CONFIGS["gemma-31b"], layers=6, vocab=8192),
                          blocks=[(1500, [40, 60, 30]), (900, []), (1200, [50, 50]), (300, [])], fp8=True,
                          dtype="bf16"),
}
CASES.update(WIDE)
#: BASELINE configuration 1's shape (2 layers, hidden 256, 4 / 2 heads of 64) through the reference's served
#: ``--fp8`` path (the backbone cast to bf16, then quantized), so the FP8 forward meets the readout bar against the
#: same path it replaces; the float32 ``--fp8`` run is stored beside it.
CASES.update({
    "qwen_tiny_fp8_served": dict(spec=CONFIGS["tiny"], lengths=("uniform", 16, 32, 160), markers=(1, 4), fp8=True,
                                 dtype="bf16"),
    "gemma_tiny_fp8_served": dict(spec=Spec("gemma", 6, 256, 4, 2, 64, 512, 4096, window=16, logit_cap=30.0),
                                  lengths=("uniform", 16, 8, 96), markers=(1, 1), fp8=True, dtype="bf16"),
    # Qwen3.5 joint layouts with images (families/qwen/packed.py:158-165, :186): image-token runs whose embeddings
    # the given features replace, and the reference's own M-RoPE positions (model/packed.py:64-70, the backbone's
    # get_rope_index over each image's (1, h, w) grid, merged 2 x 2); two sequences with images, one without
    "qwen_images": dict(spec=dataclasses.replace(CONFIGS["tiny"], mrope_section=(12, 10, 10)),
                        lengths=("list", 90, 70, 120), markers=(2, 4), fp8=False,
                        joint_images=[(20, 4, 6), (50, 2, 4), (100, 6, 4), (130, 4, 4)]),
})


#: FP8 cases also record, for layer 0, each quantized projection's input (e4m3 values and row scales) and output: the
#: per-projection pin of the FP8 arithmetic (a random deep model amplifies single e4m3 rounding flips, so the end-to-end
#: FP8 forward is compared only loosely, as the reference's own tests do: tests/gpu/test_fp8.py:4-5).
PINNED = ("q_proj", "o_proj", "gate_proj", "down_proj")
PIN_ROWS = 48
#: Rows pinned in the full-width bf16 FP8 cases (e4m3 inputs as their bytes, bf16 outputs as their bits).
WIDE_PIN_ROWS = 16


def _record_fp8(stack: contextlib.ExitStack, module, captured: dict) -> None:
    """Wraps ``module.Fp8Linear.forward`` to keep the first call's input and output of each layer-0 projection."""
    original = module.Fp8Linear.forward

    def forward(self, x):
        out = original(self, x)
        name = getattr(self, "_pin_name", None)
        if name is not None and name not in captured:
            if type(x).__name__ == "Quantized":
                values, scale = x.values, x.scale
            else:
                values, scale = module.to_e4m3(x.reshape(-1, x.shape[-1]))
            if out.dtype == torch.bfloat16:  # the served bf16 path at full width: a few rows, kept as raw bits
                rows = WIDE_PIN_ROWS
                captured[name] = (values.reshape(-1, values.shape[-1])[:rows].view(torch.uint8).numpy(),
                                  scale.float().reshape(-1)[:rows].numpy(),
                                  out.reshape(-1, out.shape[-1])[:rows].view(torch.int16).numpy().view(np.uint16))
            else:
                rows = PIN_ROWS  # the first rows suffice for the pin and keep the fixture small
                captured[name] = (values.float().reshape(-1, values.shape[-1])[:rows].numpy(),
                                  scale.float().reshape(-1)[:rows].numpy(),
                                  out.float().reshape(-1, out.shape[-1])[:rows].numpy())
        return out

    stack.enter_context(_patched(module.Fp8Linear, "forward", forward))


def _name_pins(packed, module) -> None:
    for name, child in packed.layers[0].named_modules():
        if isinstance(child, module.Fp8Linear) and name.rsplit(".", 1)[-1] in PINNED:
            child._pin_name = name.rsplit(".", 1)[-1]


def reference_forward(case: dict, spec: Spec, weights: dict, arrays: dict, seqs: list, features, dtype: str,
                      record: bool = True):
    """(hidden, logits, layer-0 FP8 pins) of the reference's own forward over ``seqs``: the backbone in float32, or
    cast to bf16 with ``dtype="bf16"`` (the reference's served precision); FP8 cases quantize it with the reference's
    own ``quantize`` after the cast, as ``--fp8`` does at load."""
    from karpo_decision.model.packed import pack
    from karpo_decision.model.readout import Readout

    head = Readout.from_rows(to_torch(weights, "readout"), cap=spec.logit_cap)
    cast = torch.bfloat16 if dtype == "bf16" else torch.float32
    captured: dict = {}
    with torch.inference_mode(), contextlib.ExitStack() as stack:
        if case["fp8"]:
            stack.enter_context(_patched(torch, "_scaled_mm", scaled_mm_contract))
        if spec.family == "qwen":
            from karpo_decision.families.qwen import packed as qp

            model = to_dtype(qwen_backbone(spec, weights), cast)
            stack.enter_context(_patched(qp, "_kernels", lambda: (delta_rule_contract, varlen_contract,
                                                                   conv_contract)))
            if features is not None:  # the vision tower's output, given
                given = torch.from_numpy(arrays["image_features"]).to(cast)
                stack.enter_context(_patched(model, "get_image_features",
                                             lambda *_, **__: types.SimpleNamespace(pooler_output=[given])))
            packed = qp.Packed(model, spec.attention)
            if case["fp8"]:
                from karpo_decision.serve import qwen_fp8
                qwen_fp8.quantize(packed)
                if record:
                    _name_pins(packed, qwen_fp8)
                    _record_fp8(stack, qwen_fp8, captured)
            p = pack(seqs, model, torch.device("cpu"))
            if p.rope is not None and features is not None:
                captured["rope"] = p.rope
        else:
            from karpo_decision.families.gemma import packed as gp
            from karpo_decision.families.gemma import sliding_attention

            lm = to_dtype(gemma_lm(spec, weights), cast)
            stack.enter_context(_patched(sliding_attention, "varlen_attn", varlen_contract))
            stack.enter_context(_patched(gp, "sdpa_kernel", lambda *_: contextlib.nullcontext()))
            backbone = types.SimpleNamespace(language_model=lm, config=types.SimpleNamespace(image_token_id=IMAGE_TOKEN))
            if features is not None:  # the vision encoder's output, given
                given = torch.from_numpy(arrays["image_features"]).to(cast)
                stack.enter_context(_patched(gp.vision, "embed", lambda *_: given))
            packed = gp.Packed(backbone, spec.attention)
            if case["fp8"]:
                from karpo_decision.serve import fp8
                stack.enter_context(_patched(fp8, "to_e4m3", fp8._rows_e4m3))
                stack.enter_context(_patched(fp8, "norm_e4m3", fp8._norm_e4m3))
                stack.enter_context(_patched(fp8, "gelu_mul_e4m3", fp8._gelu_mul_e4m3))
                fp8.quantize(packed)
                if record:
                    _name_pins(packed, fp8)
                    _record_fp8(stack, fp8, captured)
            p = pack(seqs, None, torch.device("cpu"))
        hidden = packed(p)
        logits = head(hidden)
    return hidden, logits, captured


def run_case(name: str, case: dict, seed: int = 0) -> dict[str, np.ndarray]:
    spec: Spec = case["spec"]
    weights = numpy_weights(spec, seed)
    if "blocks" in case:
        arrays = synthetic_block_arrays(case["blocks"], spec.vocab, seed + 1)
    else:
        kind, *rest = case["lengths"]
        if kind == "list":
            lengths = [int(x) for x in rest]
        elif kind == "log":  # (total, low, high[, lengths seed])
            total, low, high, *draw = rest
            lengths = synthetic_lengths(total, low, high, draw[0] if draw else seed, log_uniform=True)
        else:
            n, low, high = rest
            rng = np.random.default_rng(seed)
            lengths = [int(x) for x in rng.integers(low, high + 1, size=n)]
        arrays = synthetic_pack_arrays(lengths, spec.vocab, seed + 1, case["markers"])
    features = None
    if "images" in case:  # soft tokens (id vocab - 1) over the given (row, length) runs, and their features
        arrays = dict(arrays, input_ids=arrays["input_ids"].copy())
        arrays["input_ids"][arrays["input_ids"] == IMAGE_TOKEN] = 0
        for row, length in case["images"]:
            arrays["input_ids"][row:row + length] = IMAGE_TOKEN
        n_soft = sum(length for _, length in case["images"])
        features = np.random.default_rng(seed + 2).standard_normal((n_soft, spec.hidden)).astype(np.float32) * 0.3
        arrays["image_features"] = oracle_bf16(features)
    if "joint_images" in case:  # Qwen: an image of grid (1, gh, gw) is gh * gw / 4 image tokens from `row` on
        arrays = dict(arrays, input_ids=arrays["input_ids"].copy())
        arrays["input_ids"][arrays["input_ids"] == IMAGE_TOKEN] = 0
        rows, grids, n_soft = [], [], 0
        for row, gh, gw in case["joint_images"]:
            tokens = gh * gw // 4
            arrays["input_ids"][row:row + tokens] = IMAGE_TOKEN
            rows.append(row)
            grids.append((1, gh, gw))
            n_soft += tokens
        arrays["image_rows"], arrays["image_grids"] = np.asarray(rows), np.asarray(grids)
        features = np.random.default_rng(seed + 2).standard_normal((n_soft, spec.hidden)).astype(np.float32) * 0.3
        arrays["image_features"] = oracle_bf16(features)
        features = arrays["image_features"]
    seqs = encoded(arrays, blocks=spec.family == "gemma")
    if features is not None and spec.family == "gemma":  # sequences with soft tokens carry (placeholder) pixels
        seqs = [dataclasses.replace(q, pixel_values=torch.zeros(1, 1), image_position_ids=torch.zeros(1, 1, 2))
                if bool((q.input_ids == IMAGE_TOKEN).any()) else q for q in seqs]
    hidden, logits, captured = reference_forward(case, spec, weights, arrays, seqs, features, case.get("dtype", "fp32"))
    noise = {}
    if case.get("dtype", "fp32") == "bf16":  # the float32 run of the same case, the noise reference
        h32, l32, _ = reference_forward(case, spec, weights, arrays, seqs, features, "fp32", record=False)
        noise = {"hidden_fp32": h32.float().numpy(), "logits_fp32": l32.float().numpy()}
    rope = captured.pop("rope", None)
    pins = {}
    for proj, (values, scale, out) in captured.items():
        if values.dtype == np.uint8:  # full width, served bf16 path
            pins[f"wpin_{proj}_in_e4m3"], pins[f"wpin_{proj}_scale"], pins[f"wpin_{proj}_out_bf16"] = values, scale, out
        else:
            pins[f"pin_{proj}_in"], pins[f"pin_{proj}_scale"], pins[f"pin_{proj}_out"] = values, scale, out
    extra = {k: arrays[k] for k in ("segment_ids", "image_features") if k in arrays}
    if rope is not None:
        extra["rope"] = rope.reshape(rope.shape[0], -1).numpy()
    return {
        **pins, **extra, **noise,
        "input_ids": arrays["input_ids"], "seqpos": arrays["seqpos"], "cu": arrays["cu"],
        "markers": arrays["markers"], "marker_cu": arrays["marker_cu"],
        "hidden": hidden.float().numpy(), "logits": logits.float().numpy(),
        "seed": np.array(seed), "weights_sha256": np.array(weights_digest(weights)),
        "spec": np.array(repr(spec.as_dict())), "dtype": np.array(case.get("dtype", "fp32")),
    }


@contextlib.contextmanager
def _patched(obj, name, value):
    old = getattr(obj, name)
    setattr(obj, name, value)
    try:
        yield
    finally:
        setattr(obj, name, old)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True, help="root of a karpo-decision checkout")
    parser.add_argument("--cases", nargs="*", default=list(CASES))
    args = parser.parse_args()
    import_reference(args.reference)
    torch.manual_seed(0)
    for name in args.cases:
        out = run_case(name, CASES[name])
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(name, "tokens", len(out["input_ids"]), "markers", len(out["markers"]), "hidden", out["hidden"].shape,
              "logit range", float(np.abs(out["logits"]).max()))


if __name__ == "__main__":
    main()
