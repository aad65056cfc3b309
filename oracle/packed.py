"""numpy restatement of the reference's packed forward (Qwen-shaped and Gemma-shaped decoders) and readout.

Test infrastructure only (the checker and the timed CPU baseline); the product path never imports it.

Two modes:
- ``"fp32"``: float32 everywhere, no intermediate rounding (the reference run in float32 on CPU, which the golden
  fixtures hold);
- ``"bf16"``: float32 arithmetic with a bf16 rounding wherever the reference's bf16 path stores a bf16 tensor: after
  every projection, norm, rotation, activation product, residual sum and attention output, and for the rotary tables.
  Pointwise groups that the reference fuses into one compiled kernel (families/qwen/fused.py:51-71,
  families/gemma/fused.py:64-78) round once, at their output.

Weights are dicts of float32 arrays laid out like the Transformers modules the reference wraps (nn.Linear weights
(out, in)); ``pack`` is a dict with ``input_ids`` (T,), ``seqpos`` (T,), ``cu`` (n + 1,), ``markers`` (M,).
"""

from __future__ import annotations

import math

import numpy as np

E4M3_MAX = 448.0


# ------------------------------------------------------------------------------------------------ rounding


def bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16, returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(x.shape)


def _round(x: np.ndarray, mode: str) -> np.ndarray:
    return bf16(x) if mode == "bf16" else x.astype(np.float32, copy=False)


def _e4m3_table() -> np.ndarray:
    """Every non-negative finite e4m3fn value (bias 7, no infinities, 0x7F is NaN), ascending."""
    vals = []
    for code in range(0x7F):
        e, m = code >> 3, code & 7
        vals.append(m / 8.0 * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7))
    return np.array(vals, dtype=np.float64)


_E4M3 = _e4m3_table()


def e4m3(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float -> e4m3fn (saturating inputs are clamped to +-448 by the callers), as float32."""
    x = np.asarray(x, dtype=np.float64)
    a = np.minimum(np.abs(x), E4M3_MAX)
    idx = np.searchsorted(_E4M3, a)  # first table value >= a
    hi = _E4M3[np.minimum(idx, len(_E4M3) - 1)]
    lo = _E4M3[np.maximum(idx - 1, 0)]
    pick_lo = (a - lo) < (hi - a)
    tie = (a - lo) == (hi - a)
    lo_code = np.maximum(idx - 1, 0)
    even_lo = (lo_code & 1) == 0
    out = np.where(pick_lo | (tie & even_lo), lo, hi)
    out = np.where(a == hi, hi, out)
    return (np.sign(x) * out).astype(np.float32)


def e4m3_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Each row scaled into the e4m3 range, rounded to e4m3, and its float32 scale (serve/fp8.py:21-24,
    serve/qwen_fp8.py:20-23): scale = max(amax, 1e-12) / 448, q = e4m3(clamp(x / scale, +-448))."""
    x = np.asarray(x, dtype=np.float32)
    scale = (np.maximum(np.abs(x).max(axis=-1, keepdims=True), np.float32(1e-12)) / np.float32(E4M3_MAX))
    scale = scale.astype(np.float32)
    q = e4m3(np.clip(x / scale, -E4M3_MAX, E4M3_MAX))
    return q, scale


# ------------------------------------------------------------------------------------------------ pointwise


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float, one_plus: bool) -> np.ndarray:
    """RMSNorm over the last axis in float32: Qwen's ``x * rsqrt(mean(x^2) + eps) * (1 + w)``
    (families/qwen/fused.py:17-19) or Gemma's ``x * (mean(x^2) + eps)^-0.5 * w`` / without weight
    (families/gemma/fused.py:21-26). Unrounded; the caller rounds."""
    h = x.astype(np.float32)
    ms = (h * h).mean(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps)
    # Qwen multiplies by rsqrt, Gemma by pow(., -0.5): the same value, kept in the reference's form.
    out = h * (np.float32(1.0) / np.sqrt(ms)) if one_plus else h * np.power(ms, np.float32(-0.5))
    if weight is not None:
        w = weight.astype(np.float32)
        out = out * ((np.float32(1.0) + w) if one_plus else w)
    return out.astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    return x / (np.float32(1.0) + np.exp(-x))


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """``F.gelu(x, approximate="tanh")`` (families/gemma/fused.py:37-38)."""
    return np.float32(0.5) * x * (np.float32(1.0) + np.tanh(np.float32(math.sqrt(2.0 / math.pi)) *
                                                            (x + np.float32(0.044715) * x ** 3)))


def rope_tables(positions: np.ndarray, head_dim: int, theta: float, partial: float, mode: str,
                proportional: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin (T, rot) at ``positions``: inv_freq = 1 / theta^(arange(0, rot, 2) / rot), emb = cat(f, f)
    (Transformers' default rotary embedding, as Qwen3_5TextRotaryEmbedding / Gemma4TextRotaryEmbedding compute it, and
    cast to the activations' dtype). ``proportional`` (Transformers' "proportional" rope of Gemma 4 global layers):
    rot = head_dim, the first int(partial * head_dim // 2) frequencies 1 / theta^(2i / head_dim), the rest 0 (those
    pairs stay unrotated)."""
    if proportional:
        rot = head_dim
        angles = int(partial * head_dim // 2)
        inv_freq = 1.0 / (np.float32(theta) ** (np.arange(0, 2 * angles, 2, dtype=np.float32) / np.float32(head_dim)))
        inv_freq = np.concatenate([inv_freq.astype(np.float32), np.zeros(head_dim // 2 - angles, np.float32)])
    else:
        rot = int(head_dim * partial)
        inv_freq = (1.0 / (np.float32(theta) ** (np.arange(0, rot, 2, dtype=np.float32) / np.float32(rot))))
    inv_freq = inv_freq.astype(np.float32)
    freqs = positions.astype(np.float32)[:, None] * inv_freq[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1)
    return _round(np.cos(emb), mode), _round(np.sin(emb), mode)


def mrope_tables(rope: np.ndarray, head_dim: int, theta: float, partial: float, sections, mode: str
                 ) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin (T, rot) of Qwen3.5's interleaved M-RoPE at the (3, T) positions ``rope`` (time, height, width):
    freqs per axis as rope_tables forms them, then pair i takes the height axis where i % 3 == 1 and i < 3 *
    sections[1], the width axis where i % 3 == 2 and i < 3 * sections[2], the time axis otherwise (Transformers'
    Qwen3_5TextRotaryEmbedding.apply_interleaved_mrope), emb = cat(f, f)."""
    rot = int(head_dim * partial)
    half = rot // 2
    inv_freq = (1.0 / (np.float32(theta) ** (np.arange(0, rot, 2, dtype=np.float32) / np.float32(rot)))
                ).astype(np.float32)
    freqs = rope.astype(np.float32)[:, :, None] * inv_freq[None, None, :]  # (3, T, half)
    f = freqs[0].copy()
    for axis in (1, 2):
        idx = np.arange(axis, 3 * int(sections[axis]), 3)
        idx = idx[idx < half]
        f[:, idx] = freqs[axis][:, idx]
    emb = np.concatenate([f, f], axis=-1)
    return _round(np.cos(emb), mode), _round(np.sin(emb), mode)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE on the first ``rot`` dims of (T, H, hd) (Transformers apply_rotary_pos_emb, partial rotary
    as in Qwen3.5; families/gemma/fused.py:41-45)."""
    rot = cos.shape[-1]
    xr, xp = x[..., :rot], x[..., rot:]
    half = rot // 2
    rotated = np.concatenate([-xr[..., half:], xr[..., :half]], axis=-1)
    out = xr * cos[:, None, :] + rotated * sin[:, None, :]
    return np.concatenate([out, xp], axis=-1).astype(np.float32)


# ------------------------------------------------------------------------------------------------ attention


def attention_varlen(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_q: np.ndarray, cu_k: np.ndarray, scale: float,
                     window: tuple[int, int]) -> np.ndarray:
    """The varlen attention contract (tests/test_gemma_blocks.py:28-43 in the reference): per sequence, query i sees
    key j when i + (Lk - Lq) - left <= j <= i + (Lk - Lq) + right (-1: unbounded), GQA by head groups; float32
    softmax. q (Tq, Hq, d), k/v (Tk, Hkv, d) -> (Tq, Hq, d)."""
    left, right = window
    hq, hkv = q.shape[1], k.shape[1]
    group = hq // hkv
    out = np.zeros(q.shape, dtype=np.float32)
    for s in range(len(cu_q) - 1):
        qa, qb, ka, kb = int(cu_q[s]), int(cu_q[s + 1]), int(cu_k[s]), int(cu_k[s + 1])
        if qb == qa:
            continue
        lq, lk = qb - qa, kb - ka
        i = np.arange(lq)[:, None] + (lk - lq)
        j = np.arange(lk)[None, :]
        mask = np.ones((lq, lk), dtype=bool)
        if right >= 0:
            mask &= j <= i + right
        if left >= 0:
            mask &= j >= i - left
        for h in range(hq):
            qs = q[qa:qb, h, :].astype(np.float32)
            ks = k[ka:kb, h // group, :].astype(np.float32)
            vs = v[ka:kb, h // group, :].astype(np.float32)
            scores = (qs @ ks.T) * np.float32(scale)
            scores = np.where(mask, scores, -np.inf)
            peak = scores.max(axis=-1, keepdims=True)
            peak = np.where(np.isfinite(peak), peak, 0.0)
            p = np.exp(scores - peak)
            denom = p.sum(axis=-1, keepdims=True)
            out[qa:qb, h, :] = (p @ vs) / np.where(denom > 0, denom, 1.0)
    return out


# ------------------------------------------------------------------------------------------------ projections


def linear(x: np.ndarray, w: np.ndarray, mode: str, fp8: bool = False, prequantized=None) -> np.ndarray:
    """``x @ w.T`` (nn.Linear) rounded to the activations' dtype; with ``fp8`` the rowwise-scaled e4m3 product of
    serve/fp8.py:86-101 / serve/qwen_fp8.py:38-42: (q_x @ q_w.T) * s_x * s_w (float32 accumulation, bf16 out).
    ``w`` is then the pair (q_w, s_w) and ``prequantized`` optionally the pair (q_x, s_x)."""
    if not fp8 or not isinstance(w, tuple):  # a projection left in bf16 (Qwen: fewer than 256 outputs)
        return _round(x.astype(np.float32) @ w.astype(np.float32).T, mode)
    qw, sw = w
    qx, sx = prequantized if prequantized is not None else e4m3_rows(x)
    return _round((qx @ qw.T) * sx * sw.reshape(1, -1), mode)


#: Qwen's FP8 path keeps projections with fewer outputs in bf16 (serve/qwen_fp8.py:17, :45-56).
QWEN_FP8_MIN_FEATURES = 256


def quantize_weights(weights: dict, min_features: int = 0) -> dict:
    """Every projection weight with at least ``min_features`` outputs to (e4m3 rows, (1, out) scales) as Fp8Linear
    does at load (serve/fp8.py:86-90, serve/qwen_fp8.py:27-33)."""
    out = dict(weights)
    for key, w in weights.items():
        if key.endswith(("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "in_proj_qkv",
                         "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")) and \
                w.shape[0] >= min_features:
            q, s = e4m3_rows(w)
            out[key] = (q, s.reshape(1, -1))
    return out


# ------------------------------------------------------------------------------------------------ Gated DeltaNet


def causal_conv_silu(x: np.ndarray, weight: np.ndarray, seqpos: np.ndarray) -> np.ndarray:
    """Depthwise causal convolution over rows (T, C) with taps (C, K), cut at every sequence start (a tap reaches
    back ``shift`` rows only where seqpos >= shift: families/qwen/packed.py:47-55), float32 sums, then silu: the
    convolution and activation of the Gated DeltaNet (families/qwen/packed.py:82-87, flash-linear-attention's
    causal_conv1d with cu_seqlens)."""
    taps = weight.shape[1]
    xf = x.astype(np.float32)
    out = xf * weight[:, taps - 1].astype(np.float32)[None, :]
    for shift in range(1, taps):
        shifted = np.zeros_like(xf)
        shifted[shift:] = xf[:-shift]
        out = out + shifted * (seqpos >= shift).astype(np.float32)[:, None] * \
            weight[:, taps - 1 - shift].astype(np.float32)[None, :]
    return silu(out)


def gated_delta_rule(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray, beta: np.ndarray,
                     cu: np.ndarray) -> np.ndarray:
    """The gated delta rule per sequence and head, in its recurrent form (Transformers'
    torch_recurrent_gated_delta_rule, the contract of flash-linear-attention's chunk_gated_delta_rule that
    families/qwen/packed.py:102-103 calls with use_qk_l2norm_in_kernel): q, k L2-normalized (eps 1e-6), q scaled by
    dk^-0.5, state S (dk, dv) from zero at each sequence start; per token S = S exp(g) ; d = (v - S^T k) beta ;
    S = S + k d^T ; o = S^T q. q, k (T, H, dk), v (T, H, dv), g, beta (T, H) -> (T, H, dv) float32."""
    def l2(x):
        x = x.astype(np.float32)
        return x / np.sqrt((x * x).sum(-1, keepdims=True) + np.float32(1e-6))

    q, k = l2(q) * np.float32(q.shape[-1] ** -0.5), l2(k)
    v, g, beta = v.astype(np.float32), g.astype(np.float32), beta.astype(np.float32)
    heads, dk, dv = q.shape[1], q.shape[2], v.shape[2]
    out = np.zeros((q.shape[0], heads, dv), dtype=np.float32)
    for a, b in zip(cu[:-1].tolist(), cu[1:].tolist(), strict=True):
        state = np.zeros((heads, dk, dv), dtype=np.float32)
        for t in range(a, b):
            state = state * np.exp(g[t])[:, None, None]
            kv = np.einsum("hkv,hk->hv", state, k[t])
            delta = (v[t] - kv) * beta[t][:, None]
            state = state + k[t][:, :, None] * delta[:, None, :]
            out[t] = np.einsum("hkv,hk->hv", state, q[t])
    return out


def unit_lower_inverse(a: np.ndarray, block: int = 16) -> np.ndarray:
    """(I + A)^-1 for a strictly lower-triangular square A, by blocks of ``block`` rows: each diagonal block by forward
    substitution (row i = e_i - A_i,<i times the rows above), then, block row by block row, the blocks below the
    diagonal from (I + A) T = I: T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj. The chunked delta rule's triangular solve in
    the blocked order a tensor-core kernel would follow (small diagonal inverses, then block products)."""
    c = a.shape[0]
    t = np.zeros_like(a)
    starts = list(range(0, c, block))
    spans = [slice(b, min(c, b + block)) for b in starts]
    for sp in spans:
        n = sp.stop - sp.start
        ab, d = a[sp, sp], np.eye(n, dtype=a.dtype)
        for i in range(1, n):
            d[i, :i] = -ab[i, :i] @ d[:i, :i]
        t[sp, sp] = d
    for bi in range(1, len(spans)):
        for bj in range(bi):
            acc = sum(a[spans[bi], spans[bk]] @ t[spans[bk], spans[bj]] for bk in range(bj, bi))
            t[spans[bi], spans[bj]] = -t[spans[bi], spans[bi]] @ acc
    return t


def gated_delta_rule_chunked(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray, beta: np.ndarray,
                             cu: np.ndarray, chunk: int = 64) -> np.ndarray:
    """``gated_delta_rule`` in the chunked (WY) form that flash-linear-attention's chunk_gated_delta_rule evaluates
    (the kernel families/qwen/packed.py:102-103 calls), with the same normalization and state start per sequence. Per
    chunk of at most ``chunk`` tokens of a sequence and head, G the running sum of g from the chunk's start:
        A = strictly lower part of diag(beta) (K K^T o exp(G_i - G_j)),  T = (I + A)^-1,
        U = T diag(beta) V,  W = T diag(beta exp(G)) K,  D = U - W S,
        O = diag(exp(G)) Q S + (Q K^T o exp(G_i - G_j), j <= i) D,
        S <- exp(G_last) S + (diag(exp(G_last - G)) K)^T D.
    Equal to the recurrent form up to rounding; float32 in, float32 out."""
    def l2(x):
        x = x.astype(np.float32)
        return x / np.sqrt((x * x).sum(-1, keepdims=True) + np.float32(1e-6))

    q, k = l2(q) * np.float32(q.shape[-1] ** -0.5), l2(k)
    v, g, beta = v.astype(np.float32), g.astype(np.float32), beta.astype(np.float32)
    heads, dk, dv = q.shape[1], q.shape[2], v.shape[2]
    out = np.zeros((q.shape[0], heads, dv), dtype=np.float32)
    for a, b in zip(cu[:-1].tolist(), cu[1:].tolist(), strict=True):
        for h in range(heads):
            state = np.zeros((dk, dv), dtype=np.float32)
            for c0 in range(a, b, chunk):
                c1 = min(c0 + chunk, b)
                kc, qc, vc, bc = k[c0:c1, h], q[c0:c1, h], v[c0:c1, h], beta[c0:c1, h]
                gc = np.cumsum(g[c0:c1, h], dtype=np.float32)
                n = c1 - c0
                lower = np.tril(np.ones((n, n), dtype=bool))
                # exp(G_i - G_j) for j <= i only (the upper part would overflow and is not used)
                decay = np.exp(np.where(lower, gc[:, None] - gc[None, :], -np.inf)).astype(np.float32)
                amat = np.tril(bc[:, None] * (kc @ kc.T) * decay, -1)
                tmat = unit_lower_inverse(amat)
                u = tmat @ (bc[:, None] * vc)
                w = tmat @ ((bc * np.exp(gc))[:, None] * kc)
                d = u - w @ state
                out[c0:c1, h] = (np.exp(gc)[:, None] * qc) @ state + ((qc @ kc.T) * decay) @ d
                state = np.exp(gc[-1]) * state + (kc * np.exp(gc[-1] - gc)[:, None]).T @ d
    return out


def softplus(x: np.ndarray) -> np.ndarray:
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def linear_attention(weights: dict, spec: dict, p: str, x: np.ndarray, pack: dict, mode: str,
                     fp8: bool = False) -> np.ndarray:
    """Qwen3.5's Gated DeltaNet token mixer over the pack (families/qwen/packed.py:74-106): projections, causal
    convolution + silu, decay g = -exp(A_log) softplus(a + dt_bias) and write strength beta = sigmoid(b)
    (fused.py:42-44), query/key heads repeated to the value heads, the gated delta rule, the gated RMSNorm
    weight * bf16(norm(core)) * silu(z) (fused.py:28-31, Qwen3_5RMSNormGated) and the output projection."""
    la = p + "linear_attn."
    t = x.shape[0]
    nk, nv, dk, dv = spec["lin_k_heads"], spec["lin_v_heads"], spec["lin_k_dim"], spec["lin_v_dim"]
    kd = nk * dk
    mixed = linear(x, weights[la + "in_proj_qkv"], mode, fp8)
    z = linear(x, weights[la + "in_proj_z"], mode, fp8).reshape(t, nv, dv)
    b = linear(x, weights[la + "in_proj_b"], mode, fp8)
    a = linear(x, weights[la + "in_proj_a"], mode, fp8)
    mixed = _round(causal_conv_silu(mixed, weights[la + "conv1d"], pack["seqpos"]), mode)
    q = mixed[:, :kd].reshape(t, nk, dk)
    k = mixed[:, kd:2 * kd].reshape(t, nk, dk)
    v = mixed[:, 2 * kd:].reshape(t, nv, dv)
    g = -np.exp(weights[la + "A_log"].astype(np.float32)) * softplus(a + weights[la + "dt_bias"].astype(np.float32))
    beta = _round(np.float32(1.0) / (np.float32(1.0) + np.exp(-b)), mode)
    if nv > nk:
        q, k = np.repeat(q, nv // nk, axis=1), np.repeat(k, nv // nk, axis=1)
    core = _round(gated_delta_rule(q, k, v, g, beta, pack["cu"]), mode)
    normed = _round(core / np.sqrt((core * core).mean(-1, keepdims=True) + np.float32(spec["eps"])), mode)
    normed = _round(weights[la + "norm"].astype(np.float32) * normed, mode)
    out = _round(normed * silu(z), mode).reshape(t, nv * dv)
    return linear(out, weights[la + "out_proj"], mode, fp8)


# ------------------------------------------------------------------------------------------------ Qwen-shaped


def qwen_forward(weights: dict, spec: dict, pack: dict, mode: str = "fp32", fp8: bool = False) -> np.ndarray:
    """(M, hidden) final-normed hidden states at the markers: families/qwen/packed.py:178-187 over full-attention
    layers (``layer`` :149-156, ``full_attention`` :119-125, ``_qkv`` :108-117, ``head`` :173-176), causal window
    (-1, 0) (:31-32). With ``fp8``, every projection is the rowwise FP8 product of serve/qwen_fp8.py:38-42 (the
    activation quantized from its bf16 value at each call). ``spec["attention"] == "bidirectional"`` widens the window
    to (-1, -1) (:31-32); the reference then runs the last layer for the marker rows only (:127-140), whose result is
    the marker rows of the whole layer, which is what this restatement computes (pinned by the ``qwen_bidir``
    fixture). Joint layouts with images (``pack["image_features"]``, ``pack["image_token"]``, ``pack["rope"]``): the
    features replace the image tokens' embeddings in order (:161-165) and RoPE takes the M-RoPE positions (:186)."""
    eps, hq, hkv, hd = spec["eps"], spec["heads"], spec["kv_heads"], spec["head_dim"]
    if fp8:
        weights = quantize_weights(weights, QWEN_FP8_MIN_FEATURES)
    ids, seqpos, cu = pack["input_ids"], pack["seqpos"], pack["cu"]
    t = len(ids)
    h = _round(weights["embed_tokens"][ids], mode)  # :158-159
    if pack.get("image_features") is not None:  # :161-165 masked_scatter, features cast to the activations' dtype
        h = h.copy()
        h[ids == pack["image_token"]] = _round(pack["image_features"].astype(np.float32), mode)
    if pack.get("rope") is not None:  # :186 with Pack.rope
        cos, sin = mrope_tables(np.asarray(pack["rope"]).reshape(3, -1), hd, spec["rope_theta"],
                                spec.get("partial_rotary", 1.0), spec["mrope_section"], mode)
    else:
        cos, sin = rope_tables(seqpos, hd, spec["rope_theta"], spec.get("partial_rotary", 1.0), mode)  # :186
    window = (-1, 0) if spec.get("attention", "causal") == "causal" else (-1, -1)
    every = spec.get("full_every", 0)
    for i in range(spec["layers"]):
        p = f"layers.{i}."
        x = _round(rms_norm(h, weights[p + "input_layernorm"], eps, True), mode)  # :150
        if every and (i + 1) % every:  # a Gated DeltaNet layer (:152-153)
            a = linear_attention(weights, spec, p, x, pack, mode, fp8)
            h = _round(h + a, mode)
            y = _round(rms_norm(h, weights[p + "post_attention_layernorm"], eps, True), mode)
            g = linear(y, weights[p + "gate_proj"], mode, fp8)
            u = linear(y, weights[p + "up_proj"], mode, fp8)
            m = _round(silu(g) * u, mode)
            h = _round(h + linear(m, weights[p + "down_proj"], mode, fp8), mode)
            continue
        qg = linear(x, weights[p + "q_proj"], mode, fp8).reshape(t, hq, 2 * hd)  # :113
        q, gate = qg[..., :hd], qg[..., hd:].reshape(t, hq * hd)
        q = _round(rms_norm(q, weights[p + "q_norm"], eps, True), mode)  # :114
        k = linear(x, weights[p + "k_proj"], mode, fp8).reshape(t, hkv, hd)
        k = _round(rms_norm(k, weights[p + "k_norm"], eps, True), mode)  # :115
        v = linear(x, weights[p + "v_proj"], mode, fp8).reshape(t, hkv, hd)  # :116
        q, k = _round(apply_rope(q, cos, sin), mode), _round(apply_rope(k, cos, sin), mode)  # :121
        o = _round(attention_varlen(q, k, v, cu, cu, hd ** -0.5, window), mode).reshape(t, hq * hd)  # :123-124
        o = _round(o * (np.float32(1.0) / (np.float32(1.0) + np.exp(-gate))), mode)  # :125 sigmoid_mul
        a = linear(o, weights[p + "o_proj"], mode, fp8)  # :125
        h = _round(h + a, mode)  # :155 add_rms_norm
        y = _round(rms_norm(h, weights[p + "post_attention_layernorm"], eps, True), mode)
        g = linear(y, weights[p + "gate_proj"], mode, fp8)  # fused.mlp :95-97
        u = linear(y, weights[p + "up_proj"], mode, fp8)
        m = _round(silu(g) * u, mode)
        h = _round(h + linear(m, weights[p + "down_proj"], mode, fp8), mode)  # :156
    return _round(rms_norm(h[pack["markers"]], weights["norm"], eps, True), mode)  # head :173-176


# ------------------------------------------------------------------------------------------------ Gemma-shaped


def gemma_layer_types(spec: dict) -> list[str]:
    """Every ``global_every``-th layer global, and the last one (Transformers' Gemma4TextConfig forces a global last
    layer, the one the reference's bidirectional pruning needs: families/gemma/packed.py:172-173)."""
    every, n = spec.get("global_every", 6), spec["layers"]
    return ["full_attention" if (i + 1) % every == 0 or i == n - 1 else "sliding_attention" for i in range(n)]


def block_plan(cu: np.ndarray, segment_ids: np.ndarray, window: int) -> dict:
    """The virtual sequences of a pack of block layouts (families/gemma/packed.py:103-151): per sequence its shared
    block (queries and keys: the shared rows), then each branch (queries: the branch rows; keys: the whole shared block
    then the branch rows for global layers, the shared block's last window - 1 rows then the branch rows for sliding
    layers). Returns query bounds and, per layer kind, the key rows gathered in order with their bounds."""
    q_cu, g_rows, g_cu, s_rows, s_cu = [0], [], [0], [], [0]
    for a, b in zip(cu[:-1].tolist(), cu[1:].tolist(), strict=True):
        seg = np.asarray(segment_ids[a:b])
        change = (np.flatnonzero(seg[1:] != seg[:-1]) + 1).tolist()
        starts, ends = [0, *change], [*change, b - a]
        labels = [int(seg[i]) for i in starts]
        if labels != list(range(len(labels))):
            raise ValueError(f"segments {labels} are not a shared block followed by branches 1, 2, ...")
        shared = ends[0]
        own = np.arange(a, a + shared)
        tail = own[max(0, shared - (window - 1)):]
        q_cu.append(a + shared)
        g_rows.append(own)
        s_rows.append(own)
        g_cu.append(g_cu[-1] + shared)
        s_cu.append(s_cu[-1] + shared)
        for start, end in zip(starts[1:], ends[1:], strict=True):
            rows = np.arange(a + start, a + end)
            q_cu.append(a + end)
            g_rows.append(np.concatenate([own, rows]))
            s_rows.append(np.concatenate([tail, rows]))
            g_cu.append(g_cu[-1] + shared + len(rows))
            s_cu.append(s_cu[-1] + len(tail) + len(rows))
    return {"q_cu": np.array(q_cu), "g_rows": np.concatenate(g_rows), "g_cu": np.array(g_cu),
            "s_rows": np.concatenate(s_rows), "s_cu": np.array(s_cu)}


def image_spans(pack: dict, window: int) -> list[tuple[int, int, np.ndarray]]:
    """Per image (a run of soft-token rows ``pack["image_token"]``): (s, e, the rows its queries may see) as
    families/gemma/vision.py:174-196 plans them: in a shared (or only) block the rows before it within the window,
    in a branch the shared block's rows within the window by position and the branch's rows before it; then the
    image itself."""
    ids, cu, pos = pack["input_ids"], pack["cu"].tolist(), pack["seqpos"]
    seg = pack.get("segment_ids")
    seg = np.zeros(len(ids), dtype=np.int64) if seg is None else seg
    rows = np.flatnonzero(ids == pack["image_token"])
    breaks = (np.flatnonzero(rows[1:] != rows[:-1] + 1) + 1).tolist()
    out = []
    for a, b in zip([0, *breaks], [*breaks, len(rows)], strict=True):
        s, e = int(rows[a]), int(rows[b - 1]) + 1
        start = max(c for c in cu if c <= s)
        if int(seg[s]) == 0:
            seen = np.arange(max(start, s - (window - 1)), e)
        else:
            shared = int((seg[start:s] == 0).sum())
            branch = s - (int(pos[s]) - shared)
            first = min(max(0, int(pos[s]) - (window - 1)), shared)
            seen = np.concatenate([np.arange(start + first, start + shared), np.arange(branch, e)])
        out.append((s, e, seen))
    return out


def see_whole(o: np.ndarray, q: np.ndarray, k: np.ndarray, v: np.ndarray, pack: dict, window: int,
              scale: float) -> np.ndarray:
    """A sliding layer's output with each image's rows recomputed (families/gemma/vision.py:199-210): query row r
    sees key row c of its ``seen`` rows when position(c) >= position(r) - (window - 1), its whole image included."""
    pos = pack["seqpos"]
    out = o.copy()
    group = q.shape[1] // k.shape[1]
    for s, e, seen in image_spans(pack, window):
        mask = pos[seen][None, :] >= pos[s:e][:, None] - (window - 1)
        for h in range(q.shape[1]):
            scores = (q[s:e, h].astype(np.float32) @ k[seen, h // group].astype(np.float32).T) * np.float32(scale)
            scores = np.where(mask, scores, -np.inf)
            p = np.exp(scores - scores.max(-1, keepdims=True))
            out[s:e, h] = (p @ v[seen, h // group].astype(np.float32)) / p.sum(-1, keepdims=True)
    return out


def gemma_forward(weights: dict, spec: dict, pack: dict, mode: str = "fp32", fp8: bool = False) -> np.ndarray:
    """(M, hidden) at the markers: families/gemma/packed.py:305-323 over single-block sequences (each virtual sequence
    is a whole sequence) or over block layouts with branches (``block_plan`` :103-151, virtual sequences whose keys
    are gathered: ``block_plan`` below). Layer :262-265: attention :228-254 (q/k norm +
    RoPE, v norm without weight, scale 1.0; sliding layers window (W-1, 0) :171, global layers causal), residual
    ``h + norm(attn)`` (fused.py:29-30), MLP ``norm(down(gelu_tanh(gate z) * up z))`` with z = norm(h) (:258-260),
    ``(h + mlp) * layer_scalar`` (fused.py:33-34). Embeddings scaled by bf16(sqrt(hidden)) (:283-285). With ``fp8``,
    the projections are serve/fp8.py's: one activation quantization per fused producer (norm, gelu-mul), o_proj's
    input quantized at its call (serve/fp8.py:57-84, :104-117). ``spec["attention"] == "bidirectional"`` makes the
    global layers non-causal (:168-170, ``_global`` with causal False); the reference's marker-only last layer
    (:267-281) equals the marker rows of the whole last layer (a marker is its virtual sequence's last token), which
    is what this restatement computes (pinned by the ``gemma_bidir`` and ``gemma_blocks_bidir`` fixtures)."""
    eps, hq, w_len = spec["eps"], spec["heads"], spec["window"]
    k_eq_v = bool(spec.get("k_eq_v", False))

    def dims(kind):  # Gemma4TextAttention: global layers' head size and (attention_k_eq_v) key/value heads
        if kind != "full_attention":
            return spec["head_dim"], spec["kv_heads"]
        hkv = (spec.get("global_kv_heads") or spec["kv_heads"]) if k_eq_v else spec["kv_heads"]
        return spec.get("global_head_dim") or spec["head_dim"], hkv

    if fp8:
        weights = quantize_weights(weights)
    ids, seqpos, cu = pack["input_ids"], pack["seqpos"], pack["cu"]
    t = len(ids)
    scale = np.float32(math.sqrt(spec["hidden"]))
    if mode == "bf16":
        scale = bf16(np.array([scale]))[0]
    h = _round(weights["embed_tokens"][ids] * scale, mode)
    images = pack.get("image_features")
    if images is not None:  # the vision features over the soft-token rows, unscaled (families/gemma/packed.py:316-320)
        h[ids == pack["image_token"]] = _round(images.astype(np.float32), mode)
    types = gemma_layer_types(spec)
    proportional = spec.get("global_rope", "default") == "proportional"
    tables = {
        "sliding_attention": rope_tables(seqpos, dims("sliding_attention")[0], spec["rope_theta_local"], 1.0, mode),
        "full_attention": rope_tables(seqpos, dims("full_attention")[0], spec["rope_theta"],
                                      spec.get("global_partial_rotary", 1.0) if proportional else 1.0, mode,
                                      proportional),
    }
    causal_global = spec.get("attention", "causal") == "causal"
    segs = pack.get("segment_ids")
    plan = block_plan(cu, segs, w_len) if segs is not None and np.any(segs != 0) else None

    def normed(x, w):  # the norm (and, for fp8, the quantization fused into it: serve/fp8.py:57-69, :92-99)
        y = _round(rms_norm(x, w, eps, False), mode)
        return y, (e4m3_rows(y) if fp8 else None)

    for i in range(spec["layers"]):
        p = f"layers.{i}."
        cos, sin = tables[types[i]]
        hd, hkv = dims(types[i])
        x, xq = normed(h, weights[p + "input_layernorm"])
        q = linear(x, weights[p + "q_proj"], mode, fp8, xq).reshape(t, hq, hd)
        q = _round(apply_rope(rms_norm(q, weights[p + "q_norm"], eps, False), cos, sin), mode)
        raw = linear(x, weights[p + "k_proj"], mode, fp8, xq).reshape(t, hkv, hd)
        k = _round(apply_rope(rms_norm(raw, weights[p + "k_norm"], eps, False), cos, sin), mode)
        # attention_k_eq_v: the values are the key projection itself (families/gemma/packed.py:188)
        v = raw if p + "v_proj" not in weights else linear(x, weights[p + "v_proj"], mode, fp8, xq).reshape(t, hkv, hd)
        v = _round(rms_norm(v, None, eps, False), mode)
        if types[i] == "sliding_attention":
            window = (w_len - 1, 0)
        else:
            window = (-1, 0) if causal_global else (-1, -1)
        if plan is None:
            o = attention_varlen(q, k, v, cu, cu, 1.0, window)
        else:  # branched layouts: per virtual sequence, its gathered keys (end-aligned with its queries)
            rows, k_cu = (plan["s_rows"], plan["s_cu"]) if types[i] == "sliding_attention" else \
                (plan["g_rows"], plan["g_cu"])
            o = attention_varlen(q, k[rows], v[rows], plan["q_cu"], k_cu, 1.0, window)
        if images is not None and types[i] == "sliding_attention":
            o = see_whole(o, q, k, v, pack, w_len, 1.0)
        o = _round(o, mode).reshape(t, hq * hd)
        a = linear(o, weights[p + "o_proj"], mode, fp8)
        h = _round(h + rms_norm(a, weights[p + "post_attention_layernorm"], eps, False), mode)
        z, zq = normed(h, weights[p + "pre_feedforward_layernorm"])
        g = linear(z, weights[p + "gate_proj"], mode, fp8, zq)
        u = linear(z, weights[p + "up_proj"], mode, fp8, zq)
        m = _round(gelu_tanh(g) * u, mode)
        m = linear(m, weights[p + "down_proj"], mode, fp8)
        m = rms_norm(m, weights[p + "post_feedforward_layernorm"], eps, False)
        if mode == "bf16":
            m = bf16(m)
        h = _round((h + m) * np.float32(weights[p + "layer_scalar"]), mode)
    return _round(rms_norm(h[pack["markers"]], weights["norm"], eps, False), mode)


# ------------------------------------------------------------------------------------------------ readout


def readout(hidden: np.ndarray, weight: np.ndarray, cap: float | None = None) -> np.ndarray:
    """``Readout.forward`` (model/readout.py:30-33): float32 ``hidden @ W.T``, then ``cap * tanh(logits / cap)``."""
    logits = hidden.astype(np.float32) @ weight.astype(np.float32).T
    if cap:
        logits = np.float32(cap) * np.tanh(logits / np.float32(cap))
    return logits.astype(np.float32)
