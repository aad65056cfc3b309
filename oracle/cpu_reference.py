"""The reference's plain packed forward restated in PyTorch for the host cores, float32: the timed CPU baseline of
``bench.py`` (its ``cpu_baseline`` block and its ``--impl reference`` arm). Test infrastructure like the rest of
``oracle/``: the product path never imports it.

The reference is PyTorch code whose CPU path runs on torch's multi-threaded CPU kernels; this restatement runs the same
math on the same kernels (``torch.matmul`` for every ``nn.Linear``, ``F.scaled_dot_product_attention`` per sequence
for the varlen attention contract of the reference's tests/test_gemma_blocks.py:28-43) with every host thread, so the
baseline is the reference's own arithmetic at the speed its CPU path would have. Each function cites the reference
lines it follows; ``tests/test_oracle_golden.py`` checks it against the numpy oracle and the golden fixtures.

A layer is timed alone (``layer``), so a bounded sample can cover one or two layers of a full-size pack and scale by
the layer count: every layer of a kind does the same arithmetic on the same shapes.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def _t(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)) if isinstance(x, np.ndarray) else x


def rms_norm(x: torch.Tensor, w: torch.Tensor | None, eps: float, one_plus: bool) -> torch.Tensor:
    """Qwen ``x * rsqrt(mean(x^2) + eps) * (1 + w)`` (families/qwen/fused.py:17-19), Gemma ``x * (mean(x^2) +
    eps)^-0.5 * w`` (families/gemma/fused.py:21-26)."""
    out = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    if w is not None:
        out = out * ((1.0 + w) if one_plus else w)
    return out


def rope_table(positions: torch.Tensor, rot: int, theta: float, head_dim: int | None = None,
               angles: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin (T, rot): Transformers' default rotary embedding (inv_freq 1 / theta^(2i / rot), emb = cat(f, f)), or
    Gemma 4's proportional one (``angles`` frequencies 1 / theta^(2i / head_dim), the rest 0)."""
    if angles is None:
        inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
    else:
        inv = 1.0 / (theta ** (torch.arange(0, 2 * angles, 2, dtype=torch.float32) / head_dim))
        inv = torch.cat([inv, torch.zeros(rot // 2 - angles)])
    freqs = positions.float()[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on the first ``rot`` dims of (T, H, hd) (Transformers apply_rotary_pos_emb)."""
    rot = cos.shape[-1]
    xr, xp = x[..., :rot], x[..., rot:]
    half = rot // 2
    rotated = torch.cat([-xr[..., half:], xr[..., :half]], -1)
    return torch.cat([xr * cos[:, None] + rotated * sin[:, None], xp], -1)


def attention(q, k, v, cu: list[int], scale: float, window: tuple[int, int]) -> torch.Tensor:
    """Per sequence, query i sees key j when i - left <= j <= i + right (-1 unbounded): the varlen contract with equal
    query and key bounds, by torch's CPU attention; (T, Hq, d) -> (T, Hq, d)."""
    left, right = window
    out = torch.empty_like(q)
    gqa = q.shape[1] != k.shape[1]
    for a, b in zip(cu[:-1], cu[1:], strict=True):
        if b == a:
            continue
        qs, ks, vs = (x[a:b].transpose(0, 1)[None] for x in (q, k, v))
        if left < 0 and right == 0:
            o = F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=scale, enable_gqa=gqa)
        elif left < 0 and right < 0:
            o = F.scaled_dot_product_attention(qs, ks, vs, scale=scale, enable_gqa=gqa)
        else:
            i = torch.arange(b - a)[:, None]
            j = torch.arange(b - a)[None, :]
            mask = (j >= i - left) if left >= 0 else torch.ones(b - a, b - a, dtype=torch.bool)
            if right >= 0:
                mask &= j <= i + right
            o = F.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask, scale=scale, enable_gqa=gqa)
        out[a:b] = o[0].transpose(0, 1)
    return out


class Model:
    """float32 host copies of a model's weights (``synthetic.numpy_weights`` names) and its shape ``spec`` (a dict)."""

    def __init__(self, weights: dict, spec: dict) -> None:
        plain = (spec.get("attention", "causal") == "causal" and not spec.get("full_every") and
                 not spec.get("k_eq_v") and spec.get("global_head_dim") in (None, spec["head_dim"]) and
                 spec.get("global_rope", "default") == "default")
        if not plain:
            raise NotImplementedError("the CPU baseline restates the benchmark configurations' layers: causal, "
                                      "full-attention (Qwen) or sliding/global of one head size (Gemma)")
        self.spec = spec
        self.w = {k: _t(v) for k, v in weights.items()}

    def layer_kinds(self) -> list[str]:
        s = self.spec
        if s["family"] == "qwen":
            return ["full_attention"] * s["layers"]
        return ["full_attention" if (i + 1) % s["global_every"] == 0 or i == s["layers"] - 1 else "sliding_attention"
                for i in range(s["layers"])]

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        """families/qwen/packed.py:158-159; Gemma times bf16(sqrt(hidden)) (families/gemma/packed.py:283-285)."""
        h = self.w["embed_tokens"][ids]
        if self.spec["family"] == "gemma":
            h = h * float(torch.tensor(math.sqrt(self.spec["hidden"])).bfloat16().float())
        return h

    def tables(self, seqpos: torch.Tensor) -> dict:
        s = self.spec
        if s["family"] == "qwen":
            rot = int(s["head_dim"] * s.get("partial_rotary", 1.0))
            return {"full_attention": rope_table(seqpos, rot, s["rope_theta"])}
        return {"sliding_attention": rope_table(seqpos, s["head_dim"], s["rope_theta_local"]),
                "full_attention": rope_table(seqpos, s["head_dim"], s["rope_theta"])}

    def layer(self, i: int, h: torch.Tensor, tables: dict, cu: list[int]) -> torch.Tensor:
        """Layer ``i`` over the pack: Qwen families/qwen/packed.py:108-156 (causal full attention with the sigmoid
        output gate), Gemma families/gemma/packed.py:183-265 (sandwich norms, q/k/v norms, scale 1, sliding window
        (W - 1, 0) or causal global, GeGLU, layer scalar). Single-block sequences."""
        s, w, p = self.spec, self.w, f"layers.{i}."
        eps, hq, hkv, hd = s["eps"], s["heads"], s["kv_heads"], s["head_dim"]
        t = h.shape[0]
        kind = self.layer_kinds()[i]
        cos, sin = tables[kind]
        if s["family"] == "qwen":
            x = rms_norm(h, w[p + "input_layernorm"], eps, True)
            qg = (x @ w[p + "q_proj"].T).view(t, hq, 2 * hd)
            q, gate = qg[..., :hd], qg[..., hd:].reshape(t, hq * hd)
            q = apply_rope(rms_norm(q, w[p + "q_norm"], eps, True), cos, sin)
            k = apply_rope(rms_norm((x @ w[p + "k_proj"].T).view(t, hkv, hd), w[p + "k_norm"], eps, True), cos, sin)
            v = (x @ w[p + "v_proj"].T).view(t, hkv, hd)
            o = attention(q, k, v, cu, hd ** -0.5, (-1, 0)).reshape(t, hq * hd) * torch.sigmoid(gate)
            h = h + o @ w[p + "o_proj"].T
            y = rms_norm(h, w[p + "post_attention_layernorm"], eps, True)
            return h + (F.silu(y @ w[p + "gate_proj"].T) * (y @ w[p + "up_proj"].T)) @ w[p + "down_proj"].T
        x = rms_norm(h, w[p + "input_layernorm"], eps, False)
        q = apply_rope(rms_norm((x @ w[p + "q_proj"].T).view(t, hq, hd), w[p + "q_norm"], eps, False), cos, sin)
        k = apply_rope(rms_norm((x @ w[p + "k_proj"].T).view(t, hkv, hd), w[p + "k_norm"], eps, False), cos, sin)
        v = rms_norm((x @ w[p + "v_proj"].T).view(t, hkv, hd), None, eps, False)
        window = (s["window"] - 1, 0) if kind == "sliding_attention" else (-1, 0)
        o = attention(q, k, v, cu, 1.0, window).reshape(t, hq * hd)
        h = h + rms_norm(o @ w[p + "o_proj"].T, w[p + "post_attention_layernorm"], eps, False)
        z = rms_norm(h, w[p + "pre_feedforward_layernorm"], eps, False)
        m = (F.gelu(z @ w[p + "gate_proj"].T, approximate="tanh") * (z @ w[p + "up_proj"].T)) @ w[p + "down_proj"].T
        return (h + rms_norm(m, w[p + "post_feedforward_layernorm"], eps, False)) * w[p + "layer_scalar"]

    def head(self, h: torch.Tensor, markers: torch.Tensor) -> torch.Tensor:
        """The final norm at the markers (families/qwen/packed.py:173-176, families/gemma/packed.py:297-303), then the
        readout ``hidden @ W.T`` with the optional ``cap * tanh(logits / cap)`` (model/readout.py:30-33)."""
        s = self.spec
        x = rms_norm(h[markers], self.w["norm"], s["eps"], s["family"] == "qwen")
        logits = x @ self.w["readout"].T
        cap = s.get("logit_cap")
        return cap * torch.tanh(logits / cap) if cap else logits

    def forward(self, pack: dict) -> torch.Tensor:
        """Readout logits of a pack of single-block sequences (host arrays as ``synthetic_pack_arrays`` makes)."""
        ids = torch.from_numpy(np.asarray(pack["input_ids"], dtype=np.int64))
        seqpos = torch.from_numpy(np.asarray(pack["seqpos"], dtype=np.int64))
        cu = [int(x) for x in pack["cu"]]
        tables = self.tables(seqpos)
        h = self.embed(ids)
        for i in range(self.spec["layers"]):
            h = self.layer(i, h, tables, cu)
        return self.head(h, torch.from_numpy(np.asarray(pack["markers"], dtype=np.int64)))
