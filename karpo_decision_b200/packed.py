"""The packed prefill forward on libkd_b200: a drop-in for the reference's ``families.qwen.Packed`` /
``families.gemma.Packed`` (``model(pack) -> (M, hidden)``, final-normed hidden states at the markers in pack order)
and its ``Readout``.

Per layer, on the current CUDA stream (kernel names in parentheses):

Qwen-shaped (families/qwen/packed.py:149-156)            Gemma-shaped (families/gemma/packed.py:262-265)
  x = norm(h)                        (rmsnorm)            x = norm(h)                               (rmsnorm)
  qkv = x W_qkv^T                    (gemm)               qkv = x W_qkv^T                           (gemm)
  q, k, v, gate = qk-norm + RoPE     (qkv_norm_rope)      q, k, v = q/k norm + RoPE, v norm         (qkv_norm_rope)
  o = attn(q, k, v) * sigmoid(gate)  (attention_varlen)   o = attn(q, k, v), sliding or global      (attention_varlen)
  h += o W_o^T                       (gemm, residual)     h = h + norm(o W_o^T)                     (gemm, norm_add)
  y = norm(h)                        (rmsnorm)            z = norm(h)                               (rmsnorm)
  m = silu(y W_g^T) * (y W_u^T)      (gemm, swiglu)       m = gelu(z W_g^T) * (z W_u^T)             (gemm, geglu)
  h += m W_d^T                       (gemm, residual)     h = (h + norm(m W_d^T)) * scalar          (gemm, norm_add)

then ``norm(h[markers])`` (marker_norm). With ``fp8`` every projection is an e4m3 GEMM with per-output-row weight
scales (quantized at load, serve/fp8.py:86-90) and per-token activation scales computed by the kernel that produces
the activation (rmsnorm_e4m3), as serve/fp8.py and serve/qwen_fp8.py do.

Weights are repacked once at load: q/k/v concatenated into one projection, gate and up interleaved in blocks of 128
rows (the GEMM's fused activation epilogue reads one gate and one up block per 256-wide tile).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable

import numpy as np
import torch

from . import ops
from .plan import BlockPlan, ImagePlan, block_plan, image_plan, marker_bounds
from .synthetic import Spec

#: Qwen's FP8 path keeps projections with fewer outputs in bf16 (serve/qwen_fp8.py:17).
QWEN_FP8_MIN_FEATURES = 256
GATE_BLOCK = 128


def _tensor(x: Any, device: torch.device, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x))
    return x.detach().to(device=device, dtype=dtype).contiguous()


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """(2 * I_pad, K): blocks of 128 gate rows then the matching 128 up rows (I padded to a multiple of 128 with
    zero rows, whose activation products are zero)."""
    inter, k = gate.shape
    pad = (-inter) % GATE_BLOCK
    if pad:
        gate = torch.cat([gate, gate.new_zeros(pad, k)])
        up = torch.cat([up, up.new_zeros(pad, k)])
    blocks = gate.shape[0] // GATE_BLOCK
    return torch.stack([gate.view(blocks, GATE_BLOCK, k), up.view(blocks, GATE_BLOCK, k)], 1).reshape(-1, k)


@dataclass
class Projection:
    """One projection's weight: bf16 (N, K), or e4m3 (N, K) with float32 per-row scales."""

    weight: torch.Tensor
    scale: torch.Tensor | None = None

    @property
    def fp8(self) -> bool:
        return self.scale is not None

    @staticmethod
    def of(w: torch.Tensor, fp8: bool) -> Projection:
        if not fp8:
            return Projection(w)
        q, s = ops.quantize_rows_e4m3(w)
        return Projection(q, s)


@dataclass
class Mixer:
    """A Gated DeltaNet layer's token mixer (Qwen3_5GatedDeltaNet): its input projections write one buffer of
    ``width`` columns, [q k v (conv_dim) | z (value_dim) | b (Hv) | a (Hv) | zero padding to a multiple of 32]."""

    proj: list[tuple[Projection, int, int]]  # (projection, first column, width) into the mixer buffer
    width: int
    conv: torch.Tensor  # (conv_dim, K) bf16 taps
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    norm: torch.Tensor  # the gated RMSNorm's weight (head_v_dim)


@dataclass
class Layer:
    kind: str  # "full_attention", "sliding_attention" or "linear_attention"
    input_norm: torch.Tensor
    o: Projection  # attention's o_proj, or the Gated DeltaNet's out_proj
    post_attention_norm: torch.Tensor
    gate_up: Projection
    down: Projection
    qkv: list[tuple[Projection, int, int]] | None = None  # (projection, first output column, width) into qkv
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    mixer: Mixer | None = None
    pre_feedforward_norm: torch.Tensor | None = None
    post_feedforward_norm: torch.Tensor | None = None
    scalar: torch.Tensor | None = None


@dataclass
class JointImages:
    """A Qwen joint-layout pack with images: the image-token rows its image features are written over, and the
    rotary tables of its M-RoPE positions, one row per token (``index``: each token's row)."""

    rows: torch.Tensor  # (soft tokens,) int64
    index: torch.Tensor  # (T,) int64: 0 .. T - 1
    cos: torch.Tensor  # (T, rot) float32
    sin: torch.Tensor


def mixer_width(spec: Spec) -> int:
    """Columns of a Gated DeltaNet layer's projection buffer (padded to a multiple of 32, the GEMM's N granule)."""
    width = spec.conv_dim + spec.lin_value_dim + 2 * spec.lin_v_heads
    return width + (-width) % 32


class Workspace:
    """Activation buffers for packs of up to ``capacity`` tokens (allocated once, reused by every layer and pack).
    Per-head buffers are flat, sized for the widest layer kind (Gemma's global layers may have their own head size),
    and viewed per layer."""

    def __init__(self, spec: Spec, capacity: int, device: torch.device, fp8: bool, inter_pad: int,
                 stored_qkv: bool) -> None:
        t, h = capacity, spec.hidden
        bf = dict(dtype=torch.bfloat16, device=device)
        all_kinds = set(spec.layer_types())
        kinds = all_kinds - {"linear_attention"}  # attention kinds
        q_cols = max((spec.heads * spec.attn_dims(kind)[0] for kind in kinds), default=0)
        kv_cols = max((spec.attn_dims(kind)[0] * spec.attn_dims(kind)[1] for kind in kinds), default=0)
        self.capacity = capacity
        self.sched = torch.zeros(2, dtype=torch.int32, device=device)  # the attention launches' work counter
        self.h = torch.empty(t, h, **bf)
        self.x = torch.empty(t, h, **bf)
        # the stored projection, only for layers that take the unfused QKV path
        self._qkv = torch.empty(t * max(spec.qkv_width_of(k) for k in kinds), **bf) if stored_qkv and kinds else None
        # per rotary kind, the pack's rotary factors: (rot / 2, T) contiguous, viewed from a flat buffer per pack
        self._rot_half = {kind: rotary_width(spec, kind) // 2 for kind in kinds}
        self._cs = {kind: torch.empty(half * t, dtype=torch.int32, device=device)
                    for kind, half in self._rot_half.items()}
        self._q = torch.empty(t * q_cols, **bf)
        self._k = torch.empty(t * kv_cols, **bf)
        self._v = torch.empty(t * kv_cols, **bf)
        self._gate = torch.empty(t * q_cols, **bf) if spec.family == "qwen" else None
        self._o = torch.empty(t * q_cols, **bf)
        self.a = torch.empty(t, h, **bf)
        self.m = torch.empty(t, inter_pad, **bf)
        vd = spec.lin_value_dim if "linear_attention" in all_kinds else 0
        if vd:  # Gated DeltaNet layers: projection buffer, convolution output, delta-rule output, gated norm
            self.lin = torch.empty(t, mixer_width(spec), **bf)
            self.conv = torch.empty(t, spec.conv_dim, **bf)
            self.core = torch.empty(t, vd, **bf)
            self.gn = torch.empty(t, vd, **bf)
        if fp8:
            width = max(h, q_cols, inter_pad, vd)
            self.xq = torch.empty(t * width, dtype=torch.float8_e4m3fn, device=device)
            self.xs = torch.empty(t, dtype=torch.float32, device=device)

    @staticmethod
    def _view(flat: torch.Tensor, *shape: int) -> torch.Tensor:
        return flat[: math.prod(shape)].view(*shape)

    def heads(self, spec: Spec, kind: str, rows: int) -> tuple:
        """(q (rows, Hq, hd), k, v (rows, Hkv, hd), gate (rows, Hq * hd) or None) for a layer of ``kind``."""
        hd, hkv = spec.attn_dims(kind)
        gate = None if self._gate is None else self._view(self._gate, rows, spec.heads * hd)
        return (self._view(self._q, rows, spec.heads, hd), self._view(self._k, rows, hkv, hd),
                self._view(self._v, rows, hkv, hd), gate)

    def o(self, spec: Spec, kind: str, rows: int) -> torch.Tensor:
        return self._view(self._o, rows, spec.heads * spec.attn_dims(kind)[0])

    def qkv(self, spec: Spec, kind: str, rows: int) -> torch.Tensor:
        return self._view(self._qkv, rows, spec.qkv_width_of(kind))

    def e4m3(self, rows: int, cols: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.xq[: rows * cols].view(rows, cols), self.xs[:rows]

    def cs(self, kind: str, tokens: int) -> torch.Tensor:
        half = self._rot_half[kind]
        return self._cs[kind][: half * tokens].view(half, tokens)


def rotary_width(spec: Spec, kind: str) -> int:
    """Rotated dims of a layer of ``kind`` (the rotate-half span): Qwen head_dim * partial_rotary; Gemma the whole head
    (proportional RoPE spans the head too, its unrotated pairs having frequency 0)."""
    hd = spec.attn_dims(kind)[0]
    return int(hd * spec.partial_rotary) if spec.family == "qwen" else hd


class Packed(torch.nn.Module):
    """The packed forward of a Qwen-shaped or Gemma-shaped decoder on libkd_b200 kernels (see the module docstring).

    ``Packed(spec, weights, device)``: ``weights`` named as ``synthetic.numpy_weights`` (Transformers module names);
    ``Packed.from_backbone(backbone, attention)`` takes a loaded Transformers backbone as the reference's
    ``family.Packed(backbone, attention)`` does (decider.py:35)."""

    def __init__(self, spec: Spec, weights: dict[str, Any], device: torch.device | str = "cuda",
                 attention: str | None = None, fp8: bool = False, image_token_id: int | None = None,
                 image_features: Callable[[Any], torch.Tensor] | None = None) -> None:
        super().__init__()
        #: Gemma 4 images: the soft-token id and the pack's image features ((soft tokens, hidden), images in pack
        #: order), made by the backbone's vision encoder outside this path (families/gemma/vision.py:136-144).
        self.image_token_id = image_token_id
        self.image_features = image_features
        attention = spec.attention if attention is None else attention
        if attention not in ("causal", "bidirectional"):
            raise ValueError(f"attention must be 'causal' or 'bidirectional', not {attention!r}")
        for kind in set(spec.layer_types()) - {"linear_attention"}:
            hd = spec.attn_dims(kind)[0]
            if hd not in (64, 128, 256, 512):
                raise ValueError(f"head size {hd} ({kind}) is not one of the kernels' 64, 128, 256, 512")
        self.spec = spec
        self.device = torch.device(device)
        self.attention_mode = attention
        self.fp8 = fp8
        self.family = spec.family
        self.types = spec.layer_types()
        self.window = spec.window
        #: Bidirectional checkpoints: full (Qwen) and global (Gemma) layers see their whole (virtual) sequence, and the
        #: last layer runs for the marker rows only (families/qwen/packed.py:31-32,65-67, families/gemma/packed.py:
        #: 170-173); Gemma's sliding layers stay causal.
        self.prune_last = attention == "bidirectional"
        self.full_window = (-1, -1) if self.prune_last else (-1, 0)
        if self.prune_last and self.types[-1] != "full_attention":
            raise ValueError("pruning the last layer needs a full-attention (global) last layer")
        dev = self.device
        s = spec
        self.inter_pad = s.intermediate + (-s.intermediate) % GATE_BLOCK
        self.embed_tokens = _tensor(weights["embed_tokens"], dev)
        self.norm = _tensor(weights["norm"], dev)
        self.layers: list[Layer] = []
        norm_w = (lambda key: _tensor(weights[key], dev))
        for i in range(s.layers):
            p = f"layers.{i}."
            if self.types[i] == "linear_attention":
                self.layers.append(self._linear_layer(weights, p, fp8))
                continue
            wq, wk = (_tensor(weights[p + n], dev) for n in ("q_proj", "k_proj"))
            # attention_k_eq_v: the values are the key projection itself (families/gemma/packed.py:188); the kernels'
            # layout repeats the key rows in the value columns (the same products, so bit-equal raw values)
            wv = wk if s.shares_kv(self.types[i]) else _tensor(weights[p + "v_proj"], dev)
            qkv: list[tuple[Projection, int, int]] = []
            if fp8 and s.family == "qwen" and min(wk.shape[0], wv.shape[0]) < QWEN_FP8_MIN_FEATURES:
                # Qwen keeps narrow projections in bf16: q on its own, k and v together.
                qkv.append((Projection.of(wq, wq.shape[0] >= QWEN_FP8_MIN_FEATURES), 0, wq.shape[0]))
                qkv.append((Projection.of(torch.cat([wk, wv]), False), wq.shape[0], wk.shape[0] + wv.shape[0]))
            else:
                qkv.append((Projection.of(torch.cat([wq, wk, wv]), fp8), 0, s.qkv_width_of(self.types[i])))
            gate_up, down = self._mlp_weights(weights, p)
            layer = Layer(kind=self.types[i], input_norm=norm_w(p + "input_layernorm"), qkv=qkv,
                          q_norm=norm_w(p + "q_norm"), k_norm=norm_w(p + "k_norm"),
                          o=Projection.of(_tensor(weights[p + "o_proj"], dev), fp8),
                          post_attention_norm=norm_w(p + "post_attention_layernorm"),
                          gate_up=Projection.of(gate_up, fp8), down=Projection.of(down, fp8))
            if s.family == "gemma":
                layer.pre_feedforward_norm = norm_w(p + "pre_feedforward_layernorm")
                layer.post_feedforward_norm = norm_w(p + "post_feedforward_layernorm")
                layer.scalar = _tensor(np.asarray(weights[p + "layer_scalar"]).reshape(1)
                                       if not isinstance(weights[p + "layer_scalar"], torch.Tensor)
                                       else weights[p + "layer_scalar"].reshape(1), dev)
            self.layers.append(layer)
        attention_kinds = set(self.types) - {"linear_attention"}
        self._inv_freq = {kind: self._inv_freq_of(kind) for kind in attention_kinds}
        #: Per layer kind, whether the QKV projection's epilogue does the norms and RoPE (kd_qkv_projection): width a
        #: multiple of 256, rotary width a multiple of 32, a head within one 256-wide tile; otherwise GEMM +
        #: kd_qkv_norm_rope.
        self.fused_kinds = {kind for kind in attention_kinds
                            if s.qkv_width_of(kind) % 256 == 0 and rotary_width(s, kind) % 32 == 0
                            and s.attn_dims(kind)[0] <= 256}
        self._tables: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
        self._pair_axis: torch.Tensor | None = None  # Qwen M-RoPE: the position axis of each rotary frequency pair
        self._workspace: Workspace | None = None

    def _linear_layer(self, weights: dict[str, Any], p: str, fp8: bool) -> Layer:
        """A Gated DeltaNet layer: its input projections into one buffer (Qwen's FP8 path keeps the per-head b and a
        projections, fewer than 256 outputs, in bf16: serve/qwen_fp8.py:17), the convolution taps, decay parameters,
        gated-norm weight and output projection, then the MLP as in every layer."""
        s, dev = self.spec, self.device
        la = p + "linear_attn."
        w = {n: _tensor(weights[la + n], dev) for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")}
        width = mixer_width(s)
        wide = torch.cat([w["in_proj_qkv"], w["in_proj_z"]])
        narrow = torch.cat([w["in_proj_b"], w["in_proj_a"]])
        pad = width - wide.shape[0] - narrow.shape[0]
        if pad:
            narrow = torch.cat([narrow, narrow.new_zeros(pad, narrow.shape[1])])
        if fp8:
            proj = [(Projection.of(wide, wide.shape[0] >= QWEN_FP8_MIN_FEATURES), 0, wide.shape[0]),
                    (Projection.of(narrow, False), wide.shape[0], narrow.shape[0])]
        else:
            proj = [(Projection.of(torch.cat([wide, narrow]), False), 0, width)]
        out = _tensor(weights[la + "out_proj"], dev)
        mixer = Mixer(proj=proj, width=width, conv=_tensor(weights[la + "conv1d"], dev).reshape(s.conv_dim, -1),
                      a_log=_tensor(weights[la + "A_log"], dev), dt_bias=_tensor(weights[la + "dt_bias"], dev),
                      norm=_tensor(weights[la + "norm"], dev))
        gate_up, down = self._mlp_weights(weights, p)
        return Layer(kind="linear_attention", input_norm=_tensor(weights[p + "input_layernorm"], dev),
                     o=Projection.of(out, fp8 and out.shape[0] >= QWEN_FP8_MIN_FEATURES),
                     post_attention_norm=_tensor(weights[p + "post_attention_layernorm"], dev),
                     gate_up=Projection.of(gate_up, fp8), down=Projection.of(down, fp8), mixer=mixer)

    def _mlp_weights(self, weights: dict[str, Any], p: str) -> tuple[torch.Tensor, torch.Tensor]:
        """The MLP's interleaved gate/up weight and its down weight (padded to the interleave's width)."""
        dev, s = self.device, self.spec
        gate_up = interleave_gate_up(_tensor(weights[p + "gate_proj"], dev), _tensor(weights[p + "up_proj"], dev))
        down = _tensor(weights[p + "down_proj"], dev)
        if self.inter_pad != s.intermediate:
            down = torch.cat([down, down.new_zeros(down.shape[0], self.inter_pad - s.intermediate)], 1)
        return gate_up.contiguous(), down.contiguous()

    # ---------------------------------------------------------------- construction from a Transformers backbone

    @classmethod
    def from_backbone(cls, backbone: Any, attention: str = "causal", fp8: bool = False,
                      device: torch.device | str | None = None) -> Packed:
        """From a Transformers ``Qwen3_5Model`` (full-attention and Gated DeltaNet layers) or a Gemma 4 text model, as
        the reference's ``family.Packed(backbone, attention)``; the weights are copied into the kernels' layouts on
        ``device`` (default: the backbone's device when it is a GPU, else the current GPU)."""
        lm = getattr(backbone, "language_model", backbone)
        config = lm.config
        model_type = getattr(config, "model_type", "")
        family = "gemma" if "gemma" in model_type else "qwen"
        weights: dict[str, Any] = {"embed_tokens": lm.embed_tokens.weight, "norm": lm.norm.weight}
        # Gemma reads each layer's kind from the config (families/gemma/packed.py:168); Qwen from the layer
        # (``layer_type``, or the reference's ``block_type`` alias: families/qwen/packed.py:151)
        config_kinds = list(getattr(config, "layer_types", None) or []) if family == "gemma" else []
        kinds = []
        for i, layer in enumerate(lm.layers):
            p = f"layers.{i}."
            if config_kinds:
                kind = config_kinds[i]
            else:
                kind = getattr(layer, "layer_type", None) or getattr(layer, "block_type", None) or "full_attention"
            kinds.append(kind)
            for name in ("gate_proj", "up_proj", "down_proj"):
                weights[p + name] = getattr(layer.mlp, name).weight
            weights[p + "input_layernorm"] = layer.input_layernorm.weight
            weights[p + "post_attention_layernorm"] = layer.post_attention_layernorm.weight
            if kind == "linear_attention":
                la = layer.linear_attn
                if la.conv1d.bias is not None:  # families/qwen/packed.py:77-78
                    raise ValueError("unexpected convolution bias")
                for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
                    weights[p + "linear_attn." + name] = getattr(la, name).weight
                weights[p + "linear_attn.conv1d"] = la.conv1d.weight.squeeze(1)
                weights[p + "linear_attn.A_log"] = la.A_log
                weights[p + "linear_attn.dt_bias"] = la.dt_bias
                weights[p + "linear_attn.norm"] = la.norm.weight
                continue
            a = layer.self_attn
            for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                if getattr(a, name, None) is None:
                    if name == "v_proj" and family == "gemma" and getattr(config, "attention_k_eq_v", False):
                        continue  # attention_k_eq_v: the values are the key projection
                    raise NotImplementedError(f"layer {i} has no {name}")
                weights[p + name] = getattr(a, name).weight
            weights[p + "q_norm"] = a.q_norm.weight
            weights[p + "k_norm"] = a.k_norm.weight
            if family == "gemma":
                weights[p + "pre_feedforward_layernorm"] = layer.pre_feedforward_layernorm.weight
                weights[p + "post_feedforward_layernorm"] = layer.post_feedforward_layernorm.weight
                weights[p + "layer_scalar"] = layer.layer_scalar
        heads, kv_heads = config.num_attention_heads, config.num_key_value_heads
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // heads
        if family == "qwen":
            rope = config.rope_parameters
            every = 0
            if "linear_attention" in kinds:  # the hybrid pattern: every n-th layer full attention
                every = kinds.index("full_attention") + 1 if "full_attention" in kinds else 0
            spec = Spec("qwen", len(lm.layers), config.hidden_size, heads, kv_heads, head_dim,
                        config.intermediate_size, config.vocab_size, eps=config.rms_norm_eps,
                        rope_theta=rope["rope_theta"], partial_rotary=rope.get("partial_rotary_factor", 1.0),
                        full_every=every, lin_k_heads=getattr(config, "linear_num_key_heads", 16),
                        lin_v_heads=getattr(config, "linear_num_value_heads", 32),
                        lin_k_dim=getattr(config, "linear_key_head_dim", 128),
                        lin_v_dim=getattr(config, "linear_value_head_dim", 128),
                        conv_kernel=getattr(config, "linear_conv_kernel_dim", 4), attention=attention,
                        mrope_section=tuple(rope["mrope_section"]) if rope.get("mrope_section") else None)
            if kinds != spec.layer_types():
                raise NotImplementedError(f"layer pattern {kinds} is not a full-attention layer every n-th")
        else:
            rope = config.rope_parameters
            every = 6
            full = rope["full_attention"]
            proportional = full.get("rope_type", "default") == "proportional"
            spec = Spec("gemma", len(lm.layers), config.hidden_size, heads, kv_heads, head_dim,
                        config.intermediate_size, config.vocab_size, eps=config.rms_norm_eps,
                        rope_theta=full["rope_theta"],
                        rope_theta_local=rope["sliding_attention"]["rope_theta"], window=config.sliding_window,
                        global_every=every, logit_cap=config.final_logit_softcapping,
                        global_head_dim=getattr(config, "global_head_dim", None) or head_dim,
                        global_kv_heads=getattr(config, "num_global_key_value_heads", None),
                        k_eq_v=bool(getattr(config, "attention_k_eq_v", False)),
                        global_rope="proportional" if proportional else "default",
                        global_partial_rotary=full.get("partial_rotary_factor", 1.0) if proportional else 0.25,
                        attention=attention)
            if kinds != spec.layer_types():
                raise NotImplementedError(f"layer pattern {kinds} is not 5 sliding : 1 global")
        if device is None:
            device = next(lm.parameters()).device
            if device.type != "cuda":
                device = torch.device("cuda")
        image_token = getattr(getattr(backbone, "config", None), "image_token_id", None)
        features = None
        if family == "qwen" and getattr(backbone, "visual", None) is not None:
            def features(p: Any) -> torch.Tensor:
                """Every image's embeddings in pack order, from the backbone's own vision tower, as
                families/qwen/packed.py:161-163 makes them."""
                param = next(backbone.visual.parameters())
                out = backbone.get_image_features(p.pixel_values.to(param.device, param.dtype),
                                                  p.image_grid_thw.to(param.device), return_dict=True)
                return torch.cat(list(out.pooler_output))
        if family == "gemma" and (getattr(backbone, "vision_tower", None) is not None or
                                  getattr(backbone, "embed_vision", None) is not None):
            def features(p: Any) -> torch.Tensor:
                """Every image's soft-token embeddings in order, from the backbone's own vision tower and embedder
                (or its encoder-free embedder), as families/gemma/vision.py:136-144 makes them."""
                reader = getattr(backbone, "vision_tower", None) or backbone.embed_vision
                param = next(reader.parameters())
                out = backbone.get_image_features(p.pixel_values.to(param.device, param.dtype),
                                                  p.image_position_ids.to(param.device), return_dict=True)
                return torch.cat(list(out.pooler_output))
        return cls(spec, weights, device, attention, fp8, image_token_id=image_token, image_features=features)

    # ---------------------------------------------------------------- rotary tables

    def _inv_freq_of(self, kind: str) -> torch.Tensor:
        """Transformers' inv_freq for a layer of ``kind``, computed in float32 on the host as the backbone's rotary
        module does: default RoPE 1 / theta^(2i / rot); Gemma 4's proportional RoPE (global layers) 1 / theta^(2i / hd)
        for the first int(partial * hd // 2) pairs and 0 for the rest (modeling_rope_utils proportional)."""
        s = self.spec
        rot = rotary_width(s, kind)
        if s.family == "qwen":
            theta = s.rope_theta
        else:
            theta = s.rope_theta if kind == "full_attention" else s.rope_theta_local
        if s.family == "gemma" and kind == "full_attention" and s.global_rope == "proportional":
            angles = int(s.global_partial_rotary * rot // 2)
            inv = 1.0 / (theta ** (torch.arange(0, 2 * angles, 2, dtype=torch.int64).float() / rot))
            inv = torch.cat([inv, torch.zeros(rot // 2 - angles, dtype=torch.float32)])
        else:
            inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))
        return inv.to(self.device)

    def tables(self, kind: str, positions: int) -> tuple[torch.Tensor, torch.Tensor]:
        """cos/sin tables covering positions [0, positions) (grown in powers of two)."""
        have = self._tables.get(kind)
        if have is None or have[0].shape[0] < positions:
            size = 1 << max(10, math.ceil(math.log2(max(positions, 1))))
            self._tables[kind] = ops.rope_table(self._inv_freq[kind], size)
        return self._tables[kind]

    def workspace(self, tokens: int) -> Workspace:
        if self._workspace is None or self._workspace.capacity < tokens:
            self._workspace = None
            stored = any(layer.qkv is not None and not self._fused(layer) for layer in self.layers)
            self._workspace = Workspace(self.spec, tokens, self.device, self.fp8, self.inter_pad, stored)
        return self._workspace

    # ---------------------------------------------------------------- forward

    def _project(self, proj: Projection, x: torch.Tensor, x8: tuple | None, out: torch.Tensor,
                 epilogue: int = ops.EPI_STORE, residual: torch.Tensor | None = None) -> torch.Tensor:
        if proj.fp8:
            return ops.gemm_fp8(x8[0], x8[1], proj.weight, proj.scale, out=out, epilogue=epilogue, residual=residual)
        return ops.gemm(x, proj.weight, out=out, epilogue=epilogue, residual=residual)

    def _quantized(self, ws: Workspace, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        q, s = ws.e4m3(x.shape[0], x.shape[1])
        return ops.rmsnorm_e4m3(x, None, -1, 0.0, q=q, scale=s)

    def _normed(self, ws: Workspace, h: torch.Tensor, weight: torch.Tensor, mode: int, want_bf16: bool,
                want_fp8: bool) -> tuple[torch.Tensor | None, tuple | None]:
        """norm(h) as bf16 and/or as its e4m3 quantization (one fused kernel for the latter)."""
        t = h.shape[0]
        x = ops.rmsnorm(h, weight, mode, self.spec.eps, out=ws.x[:t]) if want_bf16 else None
        x8 = None
        if want_fp8:
            q, s = ws.e4m3(t, h.shape[1])
            x8 = ops.rmsnorm_e4m3(h, weight, mode, self.spec.eps, q=q, scale=s)
        return x, x8

    def forward(self, p: Any) -> torch.Tensor:
        """(M, hidden) final-normalized hidden states at the markers, in pack order."""
        plan = self.plan(p)
        images = self.images(p)
        return self.head(self.body(p, plan, images), p, plan, images)

    def images(self, p: Any) -> ImagePlan | JointImages | None:
        """The pack's image plan (None without images). Gemma: each image's soft-token rows and the keys they see in
        the sliding layers (families/gemma/packed.py:310-315). Qwen: the image-token rows and the rotary tables of the
        pack's M-RoPE positions (families/qwen/packed.py:158-165, :186)."""
        if getattr(p, "pixel_values", None) is None:
            return None
        if self.family == "qwen":
            return self._joint_images(p)
        seg = None if p.segment_ids_cpu is None else p.segment_ids_cpu.numpy()
        return image_plan(p.input_ids.cpu().numpy(), [int(x) for x in p.cu_cpu.tolist()], seg,
                          p.seqpos.cpu().numpy(), self.image_token_id, self.window, self.device)

    def plan(self, p: Any) -> BlockPlan | None:
        """Host planning of a pack, done before any kernel is queued: the virtual sequences of branched block layouts
        (families/gemma/packed.py:103-151; None without branches) and the reference's refusals of malformed packs:
        Qwen reads joint layouts only (families/qwen/packed.py:180-181); a Gemma block's readout marker is its last
        token, one per block or branch (families/gemma/packed.py:136-143)."""
        if getattr(p, "pixel_values", None) is not None:
            if self.image_token_id is None or self.image_features is None:
                raise ValueError("a pack with images needs the model's image_token_id and image_features")
            if self.family == "qwen" and getattr(p, "rope", None) is None:
                raise ValueError("a Qwen pack with images needs its M-RoPE positions (Pack.rope)")
            if self.family == "gemma" and not self.prune_last:  # families/gemma/packed.py:311-313
                raise ValueError("images are supported on bidirectional checkpoints only, the ones the image path was "
                                 "validated on")
            if self.image_token_id is None or self.image_features is None:
                raise ValueError("a pack with images needs the model's image_token_id and image_features")
        seg = p.segment_ids_cpu
        if self.family != "gemma":
            if p.segment_ids is not None:
                raise ValueError("the Qwen family reads joint layouts, not block layouts")
            return None
        if p.cu_cpu is None:
            raise ValueError("planning a Gemma pack needs its boundaries on the host (cu_cpu)")
        markers = getattr(p, "markers_cpu", None)
        if markers is None:
            markers = p.markers.cpu()  # a device read, as the reference's block_plan makes
        if seg is not None and bool((seg != 0).any()):
            return block_plan(p.cu_cpu, seg, self.window, self.device, markers_cpu=markers)
        marker_bounds([int(x) for x in p.cu_cpu.tolist()], np.asarray(markers))
        return None

    def _joint_images(self, p: Any) -> JointImages:
        """A Qwen joint layout's image-token rows and its rotary tables, one row per token: each frequency pair at
        the position of the M-RoPE axis it reads (Pack.rope, (3, 1, T) or (3, T); model/packed.py:64-70)."""
        rope = p.rope.reshape(p.rope.shape[0], -1).to(self.device, torch.int64).contiguous()
        t = int(p.input_ids.numel())
        if rope.shape[1] != t:
            raise ValueError(f"M-RoPE positions for {rope.shape[1]} tokens in a pack of {t}")
        if self._pair_axis is None:
            self._pair_axis = torch.tensor(self.spec.pair_axes(), dtype=torch.int32, device=self.device)
        cos, sin = ops.rope_table_axes(self._inv_freq["full_attention"], rope, self._pair_axis)
        rows = torch.nonzero(p.input_ids.to(self.device) == self.image_token_id).reshape(-1)
        index = torch.arange(t, dtype=torch.int64, device=self.device)
        return JointImages(rows=rows, index=index, cos=cos, sin=sin)

    def head(self, h: torch.Tensor, p: Any, plan: BlockPlan | None = None,
             images: ImagePlan | JointImages | None = None) -> torch.Tensor:
        """(M, hidden): the final norm of the body's output at the markers (families/qwen/packed.py:173-176,
        families/gemma/packed.py:297-303); a bidirectional model first runs its last layer for the marker rows."""
        mode = ops.NORM_ONE_PLUS if self.spec.family == "qwen" else ops.NORM_WEIGHT
        if not self.prune_last:
            return ops.marker_norm(h, p.markers, self.norm, mode, self.spec.eps)
        if plan is None and p.segment_ids_cpu is not None and bool((p.segment_ids_cpu != 0).any()):
            plan = self.plan(p)
        hm = self._last_layer_at_markers(h, p, plan, images if isinstance(images, JointImages) else None)
        return ops.rmsnorm(hm, self.norm, mode, self.spec.eps)

    def body(self, p: Any, plan: BlockPlan | None = None, images: ImagePlan | JointImages | None = None
             ) -> torch.Tensor:
        """(T, hidden) hidden states after every layer the whole pack runs (all but the last in a bidirectional
        model; the workspace's residual buffer): embedding and layers, no host synchronization, so it can be captured
        in a CUDA graph when ``p``'s tensors are static. Branched block layouts need their ``plan``; packs with
        images their ``images`` (the features written at the soft-token rows, which see their whole image in the
        sliding layers)."""
        s = self.spec
        if plan is None and p.segment_ids_cpu is not None and bool((p.segment_ids_cpu != 0).any()):
            plan = self.plan(p)
        t = int(p.input_ids.numel())
        ws = self.workspace(t)
        qwen = s.family == "qwen"
        h = ops.embed(p.input_ids, self.embed_tokens, 0.0 if qwen else math.sqrt(s.hidden), out=ws.h[:t])
        joint = images if isinstance(images, JointImages) else None
        if images is not None:  # the features over the (Gemma: scaled) token embeddings at the image-token rows
            # (families/qwen/packed.py:161-165, families/gemma/packed.py:316)
            features = self.image_features(p)
            if features.shape[0] != images.rows.numel():
                raise ValueError(f"{images.rows.numel()} soft tokens for {features.shape[0]} image features")
            ops.scatter_rows(features.to(device=self.device, dtype=torch.bfloat16).contiguous(), images.rows, h)
        rope_cs: dict[str, torch.Tensor] = {}  # per rotary kind, gathered once per pack
        for layer in self.layers[:-1] if self.prune_last else self.layers:
            if layer.kind == "linear_attention":
                self._after_attention(layer, h, self._linear_mixer(layer, h, p, ws), ws)
                continue
            q, k, v, gate = self._attention_inputs(layer, h, p, ws, rope_cs, joint)
            window = (self.window - 1, 0) if layer.kind == "sliding_attention" else self.full_window
            o_buf = ws.o(s, layer.kind, t)
            if plan is None:
                o = ops.attention_varlen(q, k, v, p.cu, p.cu, int(p.max_length), self._scale, window, gate=gate,
                                         out=o_buf, sched=ws.sched)
            else:  # each virtual sequence's keys: the shared block (or its window tail), then its own rows
                rows, k_cu = (plan.s_rows, plan.s_cu) if layer.kind == "sliding_attention" else \
                    (plan.g_rows, plan.g_cu)
                kg, vg = ops.gather_rows(k, rows), ops.gather_rows(v, rows)
                o = ops.attention_varlen(q, kg, vg, plan.q_cu, k_cu, plan.max_q, self._scale, window, gate=gate,
                                         out=o_buf, sched=ws.sched)
            if isinstance(images, ImagePlan) and layer.kind == "sliding_attention":
                # each image's rows again, over the window before the image and the whole image
                # (families/gemma/vision.py:199-210)
                oi = ops.attention_varlen(ops.gather_rows(q, images.rows), ops.gather_rows(k, images.keys),
                                          ops.gather_rows(v, images.keys), images.q_cu, images.k_cu, images.max_q,
                                          self._scale, (self.window - 1, -1), sched=ws.sched)
                ops.scatter_rows(oi, images.rows, o)
            self._after_attention(layer, h, o, ws)
        return h

    @property
    def _scale(self) -> float:
        return self.spec.head_dim ** -0.5 if self.spec.family == "qwen" else 1.0

    def _fused(self, layer: Layer) -> bool:
        return layer.kind in self.fused_kinds and len(layer.qkv) == 1

    def _linear_mixer(self, layer: Layer, h: torch.Tensor, p: Any, ws: Workspace) -> torch.Tensor:
        """A Gated DeltaNet layer's token mixer before its output projection (families/qwen/packed.py:74-106): the
        input norm and projections, causal convolution + silu, the gated delta rule over the pack's sequences and the
        gated RMSNorm; returns the (T, value_dim) rows the output projection reads."""
        s = self.spec
        t = h.shape[0]
        mix = layer.mixer
        x, x8 = self._normed(ws, h, layer.input_norm, ops.NORM_ONE_PLUS, any(not pr.fp8 for pr, _, _ in mix.proj),
                             any(pr.fp8 for pr, _, _ in mix.proj))
        buf = ws.lin[:t]
        for proj, col, width in mix.proj:
            self._project(proj, x, x8, buf if width == mix.width else buf[:, col:col + width])
        seqpos = p.seqpos if p.seqpos.dtype == torch.int64 else p.seqpos.long()
        conv = ops.conv_silu(buf, mix.conv, seqpos, channels=s.conv_dim, out=ws.conv[:t])
        vd = s.lin_value_dim
        core = ops.gated_delta_rule(conv, buf[:, s.conv_dim + vd:], mix.a_log, mix.dt_bias, p.cu, s.lin_k_heads,
                                    s.lin_v_heads, s.lin_k_dim, s.lin_v_dim, out=ws.core[:t])
        return ops.gated_norm(core, buf[:, s.conv_dim:s.conv_dim + vd], mix.norm, s.lin_v_heads, s.lin_v_dim, s.eps,
                              out=ws.gn[:t])

    def _attention_inputs(self, layer: Layer, h: torch.Tensor, p: Any, ws: Workspace,
                          rope_cs: dict[str, torch.Tensor], joint: JointImages | None = None) -> tuple:
        """q, k, v (normed, rotated) and Qwen's gate for every row of ``h`` (the layer's input norm and QKV
        projection; families/qwen/packed.py:108-121, families/gemma/packed.py:183-193). ``joint``: a Qwen pack with
        images, rotated by its M-RoPE tables (a row per token, read at the token's own index)."""
        s = self.spec
        t = h.shape[0]
        qwen = s.family == "qwen"
        mode = ops.NORM_ONE_PLUS if qwen else ops.NORM_WEIGHT
        seqpos = p.seqpos if p.seqpos.dtype == torch.int64 else p.seqpos.long()
        fp8_qkv = any(proj.fp8 for proj, _, _ in layer.qkv)
        bf16_qkv = any(not proj.fp8 for proj, _, _ in layer.qkv)
        x, x8 = self._normed(ws, h, layer.input_norm, mode, bf16_qkv, fp8_qkv)
        if joint is not None:
            seqpos, cos, sin = joint.index, joint.cos, joint.sin
        else:
            cos, sin = self.tables(layer.kind, int(p.max_length))  # a position is below its sequence's length
        heads_out = ws.heads(s, layer.kind, t)
        hd, hkv = s.attn_dims(layer.kind)
        v_mode = -1 if qwen else ops.NORM_NONE
        if self._fused(layer):
            # one GEMM whose epilogue normalizes, rotates and scatters the heads (kd_qkv_projection)
            if layer.kind not in rope_cs:
                rope_cs[layer.kind] = ops.rope_gather(seqpos, cos, sin, out=ws.cs(layer.kind, t))
            proj = layer.qkv[0][0]
            a_in, sa = (x8[0], x8[1]) if proj.fp8 else (x, None)
            return ops.qkv_projection(
                a_in, proj.weight, seqpos, s.heads, hkv, hd, qwen, layer.q_norm, layer.k_norm,
                mode, v_mode, s.eps, rope_cs[layer.kind], cos.shape[1], out=heads_out, scale_a=sa,
                scale_w=proj.scale)
        qkv = ws.qkv(s, layer.kind, t)
        for proj, col, width in layer.qkv:
            self._project(proj, x, x8, qkv[:, col:col + width] if width != qkv.shape[1] else qkv)
        return ops.qkv_norm_rope(qkv, seqpos, s.heads, hkv, hd, qwen, layer.q_norm, layer.k_norm,
                                 mode, v_mode, s.eps, cos, sin, out=heads_out)

    def _after_attention(self, layer: Layer, h: torch.Tensor, o: torch.Tensor, ws: Workspace) -> None:
        """The rest of the layer, in place on the rows of ``h`` (``o``: their attention outputs): the output
        projection and residual, then the MLP (families/qwen/packed.py:153-156, families/gemma/packed.py:262-265)."""
        s = self.spec
        t = h.shape[0]
        mode = ops.NORM_ONE_PLUS if s.family == "qwen" else ops.NORM_WEIGHT
        o8 = self._quantized(ws, o) if layer.o.fp8 else None
        if s.family == "qwen":
            self._project(layer.o, o, o8, h, ops.EPI_RESIDUAL, residual=h)  # h += o W_o^T
            y, y8 = self._normed(ws, h, layer.post_attention_norm, mode, not layer.gate_up.fp8, layer.gate_up.fp8)
            m = self._project(layer.gate_up, y, y8, ws.m[:t], ops.EPI_SWIGLU)
            m8 = self._quantized(ws, m) if layer.down.fp8 else None
            self._project(layer.down, m, m8, h, ops.EPI_RESIDUAL, residual=h)  # h += m W_d^T
        else:
            a = self._project(layer.o, o, o8, ws.a[:t])
            ops.norm_add(h, a, layer.post_attention_norm, mode, s.eps, out=h)  # h = h + norm(a)
            z, z8 = self._normed(ws, h, layer.pre_feedforward_norm, mode, not layer.gate_up.fp8, layer.gate_up.fp8)
            m = self._project(layer.gate_up, z, z8, ws.m[:t], ops.EPI_GEGLU)
            m8 = self._quantized(ws, m) if layer.down.fp8 else None
            d = self._project(layer.down, m, m8, ws.a[:t])
            ops.norm_add(h, d, layer.post_feedforward_norm, mode, s.eps, scalar=layer.scalar, out=h)

    def _last_layer_at_markers(self, h: torch.Tensor, p: Any, plan: BlockPlan | None,
                               joint: JointImages | None = None) -> torch.Tensor:
        """(M, hidden) before the final norm: the last layer for the marker rows only (families/qwen/packed.py:127-140,
        families/gemma/packed.py:267-281). Every row's keys and values come from one QKV projection of ``h`` (the
        queries and gates are then read at the markers); each marker attends to every key of its sequence (Gemma: of
        its virtual sequence) without a mask; output projection and MLP run on the marker rows."""
        layer = self.layers[-1]
        ws = self.workspace(h.shape[0])
        q, k, v, gate = self._attention_inputs(layer, h, p, ws, {}, joint)
        markers = p.markers
        n = int(markers.numel())
        qm = ops.gather_rows(q, markers)
        gm = None if gate is None else ops.gather_rows(gate, markers)
        if plan is None:
            q_cu, k_cu = p.marker_cu, p.cu
        else:
            q_cu, k_cu = plan.m_cu, plan.g_cu
            k, v = ops.gather_rows(k, plan.g_rows), ops.gather_rows(v, plan.g_rows)
        max_q = int(p.max_markers) if plan is None else 1  # a virtual sequence reads out at most one marker
        o = ops.attention_varlen(qm, k, v, q_cu, k_cu, max_q, self._scale, (-1, -1), gate=gm,
                                 out=ws.o(self.spec, layer.kind, n), sched=ws.sched)
        hm = ops.gather_rows(h, markers)
        self._after_attention(layer, hm, o, ws)
        return hm


class Readout(torch.nn.Module):
    """``hidden @ weight.T`` in float32, soft-capped as ``cap * tanh(logits / cap)`` when ``cap`` is set: the
    reference's ``Readout`` (model/readout.py:12-33) on the readout kernel."""

    def __init__(self, weight: Any, cap: float | None = None, device: torch.device | str = "cuda") -> None:
        super().__init__()
        self.weight = _tensor(weight, torch.device(device), torch.float32)
        self.cap = cap

    @classmethod
    def from_reference(cls, head: Any, device: torch.device | str | None = None) -> Readout:
        """From the reference's ``Readout`` module (its rows and cap), on ``device`` (default: the head's device when
        it is a GPU, else the current GPU)."""
        if device is None:
            device = head.weight.device if head.weight.is_cuda else "cuda"
        return cls(head.weight.detach().float(), head.cap, device)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        return ops.readout(hidden.contiguous(), self.weight, self.cap)
