"""Seeded model shapes, random-init weights and packs for tests, the smoke check and the benchmark.

The model shapes are the benchmark configurations of this build: a dense GQA decoder shaped like the reference's
Qwen3.5 full-attention layers (gated queries, q/k norms, ``(1 + w)`` norms, SwiGLU; families/qwen/packed.py) or like
its Gemma 4 text layers (sandwich norms, q/k/v norms, attention scale 1, layer scalar, scaled embedding, GeGLU,
5 sliding-window : 1 global layers; families/gemma/packed.py). Weights are bf16-representable float32 arrays from a
numpy generator (small shapes) or bf16 tensors drawn on the device (full-size benchmark shapes); packs follow the
reference's ``pack`` (model/packed.py:73-105) with sequence lengths drawn uniform or log-uniform.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, replace

import numpy as np
import torch

__all__ = ["CONFIGS", "Spec", "device_weights", "numpy_weights", "synthetic_lengths", "synthetic_pack_arrays"]


@dataclass(frozen=True)
class Spec:
    """A decoder's shape. ``family`` "qwen" (Qwen3.5 full-attention layers) or "gemma" (Gemma 4 text layers)."""

    family: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6  # Qwen, Gemma global layers
    rope_theta_local: float = 1e4  # Gemma sliding layers
    partial_rotary: float = 1.0  # Qwen: rotary dims = head_dim * partial_rotary
    window: int = 1024  # Gemma sliding window (a token and window - 1 before it)
    global_every: int = 6  # Gemma: layer i is global when (i + 1) % global_every == 0
    attention: str = "causal"
    logit_cap: float | None = None
    codes: int = 3  # readout rows
    # Gemma 4 global layers (Gemma4TextAttention): their own head size, and with attention_k_eq_v no v_proj (the
    # values are the key projection, v-normed) and their own key/value head count; proportional RoPE rotates the
    # first global_partial_rotary of the head's frequency pairs and leaves the rest unrotated.
    global_head_dim: int | None = None  # None: head_dim
    global_kv_heads: int | None = None  # with k_eq_v; None: kv_heads
    k_eq_v: bool = False
    global_rope: str = "default"  # or "proportional"
    global_partial_rotary: float = 0.25
    # Qwen3.5 hybrid stacks: every full_every-th layer is full attention and the others Gated DeltaNet layers
    # (Transformers' full_attention_interval; 0: every layer full attention), with their own head shapes.
    full_every: int = 0
    lin_k_heads: int = 16
    lin_v_heads: int = 32
    lin_k_dim: int = 128
    lin_v_dim: int = 128
    conv_kernel: int = 4
    # Qwen3.5 joint layouts with images: the interleaved M-RoPE sections (time, height, width frequency pairs; their
    # sum is the rotary pairs) of Transformers' rope_parameters["mrope_section"]. None: positions on one axis only.
    mrope_section: tuple | None = None

    def as_dict(self) -> dict:
        return asdict(self)

    def pair_axes(self) -> list[int]:
        """The position axis (0 time, 1 height, 2 width) each rotary frequency pair of a Qwen full-attention layer
        reads under interleaved M-RoPE (Transformers' apply_interleaved_mrope): pair i reads height when i % 3 == 1 and
        i < 3 * sections[1], width when i % 3 == 2 and i < 3 * sections[2], time otherwise."""
        half = int(self.head_dim * self.partial_rotary) // 2
        if self.mrope_section is None:
            return [0] * half
        sections = [int(x) for x in self.mrope_section]
        if len(sections) != 3 or sum(sections) != half:
            raise ValueError(f"mrope_section {sections} must split the {half} rotary pairs into 3")
        return [1 if i % 3 == 1 and i < 3 * sections[1] else 2 if i % 3 == 2 and i < 3 * sections[2] else 0
                for i in range(half)]

    def attn_dims(self, kind: str) -> tuple[int, int]:
        """(head size, key/value heads) of a layer of ``kind``."""
        if self.family == "gemma" and kind == "full_attention":
            hkv = (self.global_kv_heads or self.kv_heads) if self.k_eq_v else self.kv_heads
            return self.global_head_dim or self.head_dim, hkv
        return self.head_dim, self.kv_heads

    def shares_kv(self, kind: str) -> bool:
        """Whether a layer of ``kind`` takes its values from the key projection (attention_k_eq_v)."""
        return self.family == "gemma" and kind == "full_attention" and self.k_eq_v

    def q_width_of(self, kind: str) -> int:
        return self.heads * self.attn_dims(kind)[0] * (2 if self.family == "qwen" else 1)

    def qkv_width_of(self, kind: str) -> int:
        """Columns of a layer's [q | k | v] projection as the kernels lay it out (a shared-key layer's v columns
        repeat its k projection)."""
        hd, hkv = self.attn_dims(kind)
        return self.q_width_of(kind) + 2 * hkv * hd

    @property
    def q_width(self) -> int:
        """Columns of the query projection (Qwen's gated q_proj emits [q | gate] per head)."""
        return self.heads * self.head_dim * (2 if self.family == "qwen" else 1)

    @property
    def qkv_width(self) -> int:
        return self.q_width + 2 * self.kv_heads * self.head_dim

    @property
    def lin_key_dim(self) -> int:
        return self.lin_k_heads * self.lin_k_dim

    @property
    def lin_value_dim(self) -> int:
        return self.lin_v_heads * self.lin_v_dim

    @property
    def conv_dim(self) -> int:
        """Channels of a Gated DeltaNet layer's causal convolution: [q | k | v]."""
        return 2 * self.lin_key_dim + self.lin_value_dim

    def layer_types(self) -> list[str]:
        if self.family == "qwen":
            if self.full_every:
                return ["linear_attention" if (i + 1) % self.full_every else "full_attention"
                        for i in range(self.layers)]
            return ["full_attention"] * self.layers
        # Every global_every-th layer is global, and so is the last (Gemma4TextConfig forces a global last layer).
        return ["full_attention" if (i + 1) % self.global_every == 0 or i == self.layers - 1 else "sliding_attention"
                for i in range(self.layers)]

    def gemm_flops_per_token(self) -> float:
        """2 * sum(K * N) over one token's projections, all layers (a shared-key layer has no value projection)."""
        h, total = self.hidden, 0
        for kind in self.layer_types():
            if kind == "linear_attention":
                total += h * (self.conv_dim + self.lin_value_dim + 2 * self.lin_v_heads) + self.lin_value_dim * h
                total += 3 * h * self.intermediate
                continue
            hd, hkv = self.attn_dims(kind)
            kv = (1 if self.shares_kv(kind) else 2) * hkv * hd
            total += h * (self.q_width_of(kind) + kv) + self.heads * hd * h + 3 * h * self.intermediate
        return 2.0 * total


#: The benchmark configurations.
CONFIGS: dict[str, Spec] = {
    "tiny": Spec("qwen", 2, 256, 4, 2, 64, 1024, 4096),
    "qwen-0.8b": Spec("qwen", 28, 1024, 16, 8, 128, 3072, 151936),
    "qwen-4b": Spec("qwen", 36, 2560, 32, 8, 128, 9728, 151936),
    "gemma-12b": Spec("gemma", 48, 3840, 16, 8, 256, 15360, 262144, logit_cap=30.0),
    "gemma-31b": Spec("gemma", 62, 5376, 32, 16, 128, 21504, 262144, logit_cap=30.0),
}


def _bf16_exact(x: np.ndarray) -> np.ndarray:
    """Rounds float32 values to bf16-representable ones (round to nearest even)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(x.shape)


def numpy_weights(spec: Spec, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Random-init weights (bf16-representable float32), named as the Transformers modules the reference wraps.
    Projections ~ N(0, std) (Transformers' initializer_range); norm weights away from their identity value so a wrong
    norm rule shows: Qwen's ``(1 + w)`` weights ~ N(0, 0.1), Gemma's ``w`` ~ 1 + N(0, 0.1); Gemma layer scalars in
    [0.8, 1.0]; readout rows ~ N(0, std)."""
    rng = np.random.default_rng(seed)
    h, hq, inter = spec.hidden, spec.heads, spec.intermediate

    def normal(*shape, scale=std):
        return _bf16_exact(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))

    def norm_weight(n, base=1.0):
        w = rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)
        return _bf16_exact(w if spec.family == "qwen" else base * (1.0 + w))

    # Gemma's attention has scale 1.0 over q/k normalized to unit RMS: with identity-like q/k norm weights a random
    # model's logits have std sqrt(head_dim) and its softmax is one-hot, chaotic under any rounding. Trained
    # checkpoints learn small q/k norm weights; the synthetic ones are scaled to head_dim^-1/4 (logit std ~ 1).
    w: dict[str, np.ndarray] = {"embed_tokens": normal(spec.vocab, h)}
    for i, kind in enumerate(spec.layer_types()):
        p = f"layers.{i}."
        if kind == "linear_attention":
            w[p + "input_layernorm"] = norm_weight(h)
            la = p + "linear_attn."
            w[la + "in_proj_qkv"] = normal(spec.conv_dim, h)
            w[la + "in_proj_z"] = normal(spec.lin_value_dim, h)
            w[la + "in_proj_b"] = normal(spec.lin_v_heads, h)
            w[la + "in_proj_a"] = normal(spec.lin_v_heads, h)
            w[la + "conv1d"] = normal(spec.conv_dim, spec.conv_kernel, scale=0.3)
            # A = exp(A_log) uniform in [1, 16]; dt_bias the inverse softplus of dt log-uniform in [1e-3, 1e-1] (the
            # usual Mamba-style initialization, so the state keeps a memory over many tokens)
            w[la + "A_log"] = _bf16_exact(np.log(rng.uniform(1.0, 16.0, spec.lin_v_heads)).astype(np.float32))
            dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), spec.lin_v_heads))
            w[la + "dt_bias"] = _bf16_exact((dt + np.log(-np.expm1(-dt))).astype(np.float32))
            w[la + "norm"] = _bf16_exact((1.0 + 0.1 * rng.standard_normal(spec.lin_v_dim)).astype(np.float32))
            w[la + "out_proj"] = normal(h, spec.lin_value_dim)
            w[p + "post_attention_layernorm"] = norm_weight(h)
            w[p + "gate_proj"] = normal(inter, h)
            w[p + "up_proj"] = normal(inter, h)
            w[p + "down_proj"] = normal(h, inter)
            continue
        hd, hkv = spec.attn_dims(kind)
        qk_base = hd ** -0.25 if spec.family == "gemma" else 1.0
        w[p + "input_layernorm"] = norm_weight(h)
        w[p + "q_proj"] = normal(spec.q_width_of(kind), h)
        w[p + "k_proj"] = normal(hkv * hd, h)
        if not spec.shares_kv(kind):
            w[p + "v_proj"] = normal(hkv * hd, h)
        w[p + "q_norm"] = norm_weight(hd, qk_base)
        w[p + "k_norm"] = norm_weight(hd, qk_base)
        w[p + "o_proj"] = normal(h, hq * hd)
        w[p + "post_attention_layernorm"] = norm_weight(h)
        w[p + "gate_proj"] = normal(inter, h)
        w[p + "up_proj"] = normal(inter, h)
        w[p + "down_proj"] = normal(h, inter)
        if spec.family == "gemma":
            w[p + "pre_feedforward_layernorm"] = norm_weight(h)
            w[p + "post_feedforward_layernorm"] = norm_weight(h)
            w[p + "layer_scalar"] = _bf16_exact(rng.uniform(0.8, 1.0, size=(1,)).astype(np.float32))
    w["norm"] = norm_weight(h)
    w["readout"] = normal(spec.codes, h)
    return w


def device_weights(spec: Spec, seed: int, device: torch.device, std: float = 0.02) -> dict[str, torch.Tensor]:
    """The same layout as ``numpy_weights`` drawn directly on ``device`` in bf16 (full-size benchmark models, where a
    host-side draw would take minutes): a torch generator seeded with ``seed`` on that device."""
    gen = torch.Generator(device=device).manual_seed(seed)
    h, hq, inter = spec.hidden, spec.heads, spec.intermediate

    def normal(*shape, scale=std):
        return (torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * scale).bfloat16()

    def norm_weight(n, base=1.0):
        w = torch.randn(n, generator=gen, device=device, dtype=torch.float32) * 0.1
        return (w if spec.family == "qwen" else base * (1.0 + w)).bfloat16()

    w: dict[str, torch.Tensor] = {"embed_tokens": normal(spec.vocab, h)}
    for i, kind in enumerate(spec.layer_types()):
        p = f"layers.{i}."
        if kind == "linear_attention":
            nv = spec.lin_v_heads
            w[p + "input_layernorm"] = norm_weight(h)
            la = p + "linear_attn."
            w[la + "in_proj_qkv"] = normal(spec.conv_dim, h)
            w[la + "in_proj_z"] = normal(spec.lin_value_dim, h)
            w[la + "in_proj_b"] = normal(nv, h)
            w[la + "in_proj_a"] = normal(nv, h)
            w[la + "conv1d"] = normal(spec.conv_dim, spec.conv_kernel, scale=0.3)
            uniform = torch.rand(nv, generator=gen, device=device)
            w[la + "A_log"] = torch.log(1.0 + 15.0 * uniform).bfloat16()
            dt = torch.exp(math.log(1e-3) + (math.log(1e-1) - math.log(1e-3)) *
                           torch.rand(nv, generator=gen, device=device))
            w[la + "dt_bias"] = (dt + torch.log(-torch.expm1(-dt))).bfloat16()
            w[la + "norm"] = (1.0 + 0.1 * torch.randn(spec.lin_v_dim, generator=gen, device=device)).bfloat16()
            w[la + "out_proj"] = normal(h, spec.lin_value_dim)
            w[p + "post_attention_layernorm"] = norm_weight(h)
            w[p + "gate_proj"] = normal(inter, h)
            w[p + "up_proj"] = normal(inter, h)
            w[p + "down_proj"] = normal(h, inter)
            continue
        hd, hkv = spec.attn_dims(kind)
        qk_base = hd ** -0.25 if spec.family == "gemma" else 1.0
        w[p + "input_layernorm"] = norm_weight(h)
        w[p + "q_proj"] = normal(spec.q_width_of(kind), h)
        w[p + "k_proj"] = normal(hkv * hd, h)
        if not spec.shares_kv(kind):
            w[p + "v_proj"] = normal(hkv * hd, h)
        w[p + "q_norm"] = norm_weight(hd, qk_base)
        w[p + "k_norm"] = norm_weight(hd, qk_base)
        w[p + "o_proj"] = normal(h, hq * hd)
        w[p + "post_attention_layernorm"] = norm_weight(h)
        w[p + "gate_proj"] = normal(inter, h)
        w[p + "up_proj"] = normal(inter, h)
        w[p + "down_proj"] = normal(h, inter)
        if spec.family == "gemma":
            w[p + "pre_feedforward_layernorm"] = norm_weight(h)
            w[p + "post_feedforward_layernorm"] = norm_weight(h)
            w[p + "layer_scalar"] = (0.8 + 0.2 * torch.rand(1, generator=gen, device=device)).bfloat16()
    w["norm"] = norm_weight(h)
    w["readout"] = normal(spec.codes, h)
    return w


def synthetic_lengths(total: int, low: int, high: int, seed: int, log_uniform: bool = True) -> list[int]:
    """Sequence lengths drawn (log-)uniform in [low, high] until they fill ``total`` tokens exactly (the last one
    truncated to fit, at least 1)."""
    rng = np.random.default_rng(seed)
    out, used = [], 0
    while used < total:
        if log_uniform:
            n = int(round(math.exp(rng.uniform(math.log(low), math.log(high)))))
        else:
            n = int(rng.integers(low, high + 1))
        n = min(n, total - used)
        out.append(n)
        used += n
    return out


def synthetic_pack_arrays(lengths: list[int], vocab: int, seed: int, markers_per_seq: tuple[int, int] = (1, 1)
                          ) -> dict[str, np.ndarray]:
    """A pack's host arrays (model/packed.py:73-105 for text-only joint sequences): ids uniform in [0, vocab),
    ``seqpos`` restarting at 0 per sequence, ``cu`` boundaries, and per sequence k markers (k uniform in
    ``markers_per_seq``): its last token plus k - 1 distinct earlier positions, sorted, as global rows."""
    rng = np.random.default_rng(seed)
    ids, seqpos, markers, marker_counts = [], [], [], []
    cu = [0]
    for n in lengths:
        ids.append(rng.integers(0, vocab, size=n, dtype=np.int64))
        seqpos.append(np.arange(n, dtype=np.int64))
        k = int(rng.integers(markers_per_seq[0], markers_per_seq[1] + 1))
        k = max(1, min(k, n))
        extra = rng.choice(n - 1, size=k - 1, replace=False) if k > 1 else np.zeros(0, dtype=np.int64)
        local = np.sort(np.concatenate([extra.astype(np.int64), np.array([n - 1], dtype=np.int64)]))
        markers.append(local + cu[-1])
        marker_counts.append(k)
        cu.append(cu[-1] + n)
    return {
        "input_ids": np.concatenate(ids),
        "seqpos": np.concatenate(seqpos),
        "cu": np.array(cu, dtype=np.int64),
        "markers": np.concatenate(markers),
        "marker_cu": np.concatenate([[0], np.cumsum(marker_counts)]).astype(np.int64),
    }


def small(spec: Spec, **changes) -> Spec:
    """``spec`` with some fields changed (test-sized variants)."""
    return replace(spec, **changes)


def synthetic_block_arrays(layouts: list[tuple[int, list[int]]], vocab: int, seed: int) -> dict[str, np.ndarray]:
    """A pack of block layouts (the reference's blocks.py:194-214): per sequence ``(shared, branches)``. A sequence
    without branches is one block: positions 0..n-1, segment 0, one marker at its last token. With branches, the
    shared block (segment 0, positions 0..shared-1) is followed by branch k (segment k, positions restarting at
    ``shared``), and each branch's last token is a marker."""
    rng = np.random.default_rng(seed)
    ids, pos, seg, markers, counts, cu = [], [], [], [], [], [0]
    for shared, branches in layouts:
        start = cu[-1]
        if not branches:
            pos.append(np.arange(shared))
            seg.append(np.zeros(shared, dtype=np.int64))
            markers.append(np.array([start + shared - 1]))
            counts.append(1)
            n = shared
        else:
            p, s, m, at = [np.arange(shared)], [np.zeros(shared, dtype=np.int64)], [], shared
            for k, length in enumerate(branches, start=1):
                p.append(np.arange(shared, shared + length))
                s.append(np.full(length, k, dtype=np.int64))
                at += length
                m.append(start + at - 1)
            pos.append(np.concatenate(p))
            seg.append(np.concatenate(s))
            markers.append(np.array(m))
            counts.append(len(branches))
            n = at
        ids.append(rng.integers(0, vocab, size=n, dtype=np.int64))
        cu.append(start + n)
    return {
        "input_ids": np.concatenate(ids), "seqpos": np.concatenate(pos).astype(np.int64),
        "segment_ids": np.concatenate(seg), "cu": np.array(cu, dtype=np.int64),
        "markers": np.concatenate(markers).astype(np.int64),
        "marker_cu": np.concatenate([[0], np.cumsum(counts)]).astype(np.int64),
    }
