"""Tensor-level wrappers over the C ABI (``_lib``): shape and dtype checks, output allocation by PyTorch, the current
stream. Each op is one entry point of libkd_b200; none has a fallback.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import EPI_GEGLU, EPI_RESIDUAL, EPI_STORE, EPI_SWIGLU, NORM_NONE, NORM_ONE_PLUS, NORM_WEIGHT, call

__all__ = ["EPI_GEGLU", "EPI_RESIDUAL", "EPI_STORE", "EPI_SWIGLU", "NORM_NONE", "NORM_ONE_PLUS", "NORM_WEIGHT",
           "add_rmsnorm", "attention_varlen", "check_status", "embed", "gather_rows", "gemm", "gemm_fp8", "marker_norm",
           "norm_add", "qkv_norm_rope", "qkv_projection", "quantize_rows_e4m3", "readout", "rmsnorm", "rmsnorm_e4m3",
           "rope_gather", "rope_table", "rope_table_axes",
           "sched_pair", "status_word"]

_STATUS: dict[int, torch.Tensor] = {}
_SCHED: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The device's int32 status word that pipelined kernels write a timeout into (zero while healthy)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _STATUS:
        _STATUS[index] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
    return _STATUS[index]


def sched_pair(device: torch.device) -> torch.Tensor:
    """The device's default int32[2] work counter for attention launches (zero between launches). Launches that can
    run at the same time (different streams, no ordering) take their own pair through ``attention_varlen(sched=)``."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _SCHED:
        _SCHED[index] = torch.zeros(2, dtype=torch.int32, device=torch.device("cuda", index))
    return _SCHED[index]


def check_status(device: torch.device) -> None:
    """Raises when a kernel on ``device`` recorded a timed-out wait (synchronizes)."""
    word = status_word(device)
    value = int(word.item())
    if value != _lib.KD_OK:
        word.zero_()
        raise _lib.KernelError(f"a libkd_b200 kernel gave up waiting on {device} (status {value})")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _rowmajor(t: torch.Tensor, name: str) -> None:
    _require(t.dim() == 2 and t.stride(1) == 1, f"{name} must be 2-D with contiguous rows")
    _require(t.is_cuda, f"{name} must be on a CUDA device")


def gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, epilogue: int = EPI_STORE,
         residual: torch.Tensor | None = None) -> torch.Tensor:
    """``epilogue(a @ w.T)`` in bf16 (a: (M, K) bf16, w: (N, K) bf16). For the gated epilogues ``w`` holds gate and
    up rows interleaved per 256 (``weights.interleave_gate_up``) and the result has N / 2 columns."""
    _rowmajor(a, "a")
    _rowmajor(w, "w")
    _require(a.dtype == torch.bfloat16 and w.dtype == torch.bfloat16, "gemm operands must be bf16")
    _require(a.shape[1] == w.shape[1], f"K mismatch: {tuple(a.shape)} x {tuple(w.shape)}")
    m, n = a.shape[0], w.shape[0]
    width = n // 2 if epilogue in (EPI_SWIGLU, EPI_GEGLU) else n
    if out is None:
        out = torch.empty(m, width, dtype=torch.bfloat16, device=a.device)
    _rowmajor(out, "out")
    if epilogue == EPI_RESIDUAL:
        _require(residual is not None, "the residual epilogue needs residual")
        _rowmajor(residual, "residual")
    call("kd_gemm_bf16", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(), out.stride(0),
         _ptr(residual), residual.stride(0) if residual is not None else 0, m, n, a.shape[1], epilogue,
         status_word(a.device).data_ptr(), _stream(a))
    return out


def gemm_fp8(a: torch.Tensor, scale_a: torch.Tensor, w: torch.Tensor, scale_w: torch.Tensor,
             out: torch.Tensor | None = None, epilogue: int = EPI_STORE,
             residual: torch.Tensor | None = None) -> torch.Tensor:
    """``epilogue((a @ w.T) * scale_a[:, None] * scale_w[None, :])`` in bf16; a (M, K) and w (N, K) e4m3, scales
    float32 (M,) and (N,) (``torch._scaled_mm`` with rowwise scales)."""
    _rowmajor(a, "a")
    _rowmajor(w, "w")
    _require(a.dtype == torch.float8_e4m3fn and w.dtype == torch.float8_e4m3fn, "gemm_fp8 operands must be e4m3")
    _require(scale_a.dtype == torch.float32 and scale_w.dtype == torch.float32, "fp8 scales must be float32")
    _require(scale_a.numel() == a.shape[0] and scale_w.numel() == w.shape[0], "one scale per row of a and of w")
    _require(scale_a.is_contiguous() and scale_w.is_contiguous(), "fp8 scales must be contiguous")
    m, n = a.shape[0], w.shape[0]
    width = n // 2 if epilogue in (EPI_SWIGLU, EPI_GEGLU) else n
    if out is None:
        out = torch.empty(m, width, dtype=torch.bfloat16, device=a.device)
    _rowmajor(out, "out")
    if epilogue == EPI_RESIDUAL:
        _require(residual is not None, "the residual epilogue needs residual")
        _rowmajor(residual, "residual")
    call("kd_gemm_fp8", a.data_ptr(), a.stride(0), scale_a.data_ptr(), w.data_ptr(), w.stride(0),
         scale_w.data_ptr(), out.data_ptr(), out.stride(0), _ptr(residual),
         residual.stride(0) if residual is not None else 0, m, n, a.shape[1], epilogue,
         status_word(a.device).data_ptr(), _stream(a))
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, scale: float = 0.0, out: torch.Tensor | None = None
          ) -> torch.Tensor:
    """``table[ids]`` (times bf16(scale) when scale != 0)."""
    _require(ids.dtype == torch.int64 and ids.is_contiguous(), "ids must be contiguous int64")
    _rowmajor(table, "table")
    t = ids.numel()
    if out is None:
        out = torch.empty(t, table.shape[1], dtype=torch.bfloat16, device=table.device)
    call("kd_embed", ids.data_ptr(), t, table.data_ptr(), table.shape[0], table.shape[1], float(scale),
         out.data_ptr(), _stream(table))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor | None, mode: int, eps: float,
            out: torch.Tensor | None = None) -> torch.Tensor:
    _rowmajor(x, "x")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    call("kd_rmsnorm", x.data_ptr(), x.stride(0), _ptr(weight), mode, float(eps), out.data_ptr(), out.stride(0),
         x.shape[0], x.shape[1], _stream(x))
    return out


def add_rmsnorm(h: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, mode: int, eps: float,
                y: torch.Tensor | None = None) -> torch.Tensor:
    """In place ``h = h + x``; returns ``norm(h)``."""
    _require(h.is_contiguous() and x.is_contiguous() and h.shape == x.shape, "h and x: same contiguous shape")
    if y is None:
        y = torch.empty_like(h)
    call("kd_add_rmsnorm", h.data_ptr(), x.data_ptr(), _ptr(weight), mode, float(eps), y.data_ptr(), h.shape[0],
         h.shape[1], _stream(h))
    return y


def norm_add(h: torch.Tensor, x: torch.Tensor, weight: torch.Tensor | None, mode: int, eps: float,
             scalar: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``h + norm(x)``, or ``(h + bf16(norm(x))) * scalar``; ``out`` may be ``h``."""
    _require(h.is_contiguous() and x.is_contiguous() and h.shape == x.shape, "h and x: same contiguous shape")
    if out is None:
        out = torch.empty_like(h)
    call("kd_norm_add", h.data_ptr(), x.data_ptr(), _ptr(weight), mode, float(eps), _ptr(scalar), out.data_ptr(),
         h.shape[0], h.shape[1], _stream(h))
    return out


def rmsnorm_e4m3(x: torch.Tensor, weight: torch.Tensor | None, mode: int, eps: float,
                 q: torch.Tensor | None = None, scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``norm(x)`` rounded to bf16 and quantized per row to e4m3 (mode < 0: no norm); returns (q, scale)."""
    _rowmajor(x, "x")
    rows, cols = x.shape
    if q is None:
        q = torch.empty(rows, cols, dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty(rows, dtype=torch.float32, device=x.device)
    call("kd_rmsnorm_e4m3", x.data_ptr(), x.stride(0), _ptr(weight), mode, float(eps), q.data_ptr(),
         scale.data_ptr(), rows, cols, _stream(x))
    return q, scale


def quantize_rows_e4m3(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row e4m3 quantization of a bf16 weight (load time): (q (rows, cols) e4m3, scale (rows,) float32)."""
    _require(x.is_contiguous() and x.dtype == torch.bfloat16, "quantize_rows_e4m3 takes contiguous bf16")
    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty(rows, dtype=torch.float32, device=x.device)
    call("kd_quantize_rows_e4m3", x.data_ptr(), rows, cols, q.data_ptr(), scale.data_ptr(), _stream(x))
    return q, scale


def rope_table(inv_freq: torch.Tensor, positions: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) float32 tables (positions, rot), bf16-rounded values; inv_freq float32 (rot / 2,) on the device."""
    _require(inv_freq.dtype == torch.float32 and inv_freq.is_contiguous(), "inv_freq: contiguous float32")
    rot = 2 * inv_freq.numel()
    cos = torch.empty(positions, rot, dtype=torch.float32, device=inv_freq.device)
    sin = torch.empty_like(cos)
    call("kd_rope_table", inv_freq.data_ptr(), rot, positions, cos.data_ptr(), sin.data_ptr(), _stream(inv_freq))
    return cos, sin


def rope_table_axes(inv_freq: torch.Tensor, positions: torch.Tensor, pair_axis: torch.Tensor
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) float32 tables (T, rot), one row per token, for M-RoPE: ``positions`` int64 (axes, T) holds each
    token's position on every axis, ``pair_axis`` int32 (rot / 2,) the axis each frequency pair reads."""
    _require(inv_freq.dtype == torch.float32 and inv_freq.is_contiguous(), "inv_freq: contiguous float32")
    _require(positions.dtype == torch.int64 and positions.dim() == 2 and positions.stride(1) == 1,
             "positions: int64 (axes, T) with contiguous rows")
    _require(pair_axis.dtype == torch.int32 and pair_axis.is_contiguous() and pair_axis.numel() == inv_freq.numel(),
             "pair_axis: contiguous int32, one entry per frequency pair")
    rot = 2 * inv_freq.numel()
    axes, t = positions.shape
    cos = torch.empty(t, rot, dtype=torch.float32, device=inv_freq.device)
    sin = torch.empty_like(cos)
    call("kd_rope_table_axes", inv_freq.data_ptr(), rot, positions.data_ptr(), positions.stride(0), t,
         pair_axis.data_ptr(), axes, cos.data_ptr(), sin.data_ptr(), _stream(inv_freq))
    return cos, sin


def qkv_norm_rope(qkv: torch.Tensor, seqpos: torch.Tensor, heads: int, kv_heads: int, head_dim: int, gated: bool,
                  q_norm: torch.Tensor | None, k_norm: torch.Tensor | None, qk_mode: int, v_mode: int, eps: float,
                  cos: torch.Tensor, sin: torch.Tensor, out: tuple | None = None) -> tuple:
    """(q (T, Hq, hd), k (T, Hkv, hd), v (T, Hkv, hd), gate (T, Hq * hd) or None) from the fused QKV output."""
    _rowmajor(qkv, "qkv")
    _require(seqpos.dtype == torch.int64 and seqpos.is_contiguous(), "seqpos must be contiguous int64")
    t = qkv.shape[0]
    dev = qkv.device
    if out is None:
        q = torch.empty(t, heads, head_dim, dtype=torch.bfloat16, device=dev)
        k = torch.empty(t, kv_heads, head_dim, dtype=torch.bfloat16, device=dev)
        v = torch.empty(t, kv_heads, head_dim, dtype=torch.bfloat16, device=dev)
        gate = torch.empty(t, heads * head_dim, dtype=torch.bfloat16, device=dev) if gated else None
    else:
        q, k, v, gate = out
    rot = cos.shape[1]
    call("kd_qkv_norm_rope", qkv.data_ptr(), qkv.stride(0), t, seqpos.data_ptr(), heads, kv_heads, head_dim,
         int(gated), _ptr(q_norm), _ptr(k_norm), qk_mode, v_mode, float(eps), cos.data_ptr(), sin.data_ptr(), rot,
         q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(gate), _stream(qkv))
    return q, k, v, gate


def attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_q: torch.Tensor, cu_k: torch.Tensor,
                     max_q: int, scale: float, window: tuple[int, int], gate: torch.Tensor | None = None,
                     out: torch.Tensor | None = None, sched: torch.Tensor | None = None) -> torch.Tensor:
    """Varlen attention (the reference's varlen contract, end-aligned window); q (Tq, Hq, d), k/v (Tk, Hkv, d),
    int32 boundaries on the device; returns (Tq, Hq * d), gated by sigmoid(gate) when given. ``sched`` is the
    launch's int32[2] work counter (default: the device's, ``sched_pair``)."""
    _require(q.dim() == 3 and k.dim() == 3 and v.dim() == 3, "q, k, v must be (rows, heads, head_dim)")
    _require(q.stride(2) == 1 and k.stride(2) == 1 and v.stride(2) == 1, "head_dim must be contiguous")
    _require(q.stride(1) == q.shape[2] and k.stride(1) == k.shape[2] and v.stride(1) == v.shape[2],
             "heads must be packed within a row")
    _require(cu_q.dtype == torch.int32 and cu_k.dtype == torch.int32, "boundaries must be int32")
    tq, hq, d = q.shape
    if sched is None:
        sched = sched_pair(q.device)
    _require(sched.dtype == torch.int32 and sched.numel() >= 2 and sched.is_contiguous(),
             "sched must be a contiguous int32 pair")
    if out is None:
        out = torch.empty(tq, hq * d, dtype=torch.bfloat16, device=q.device)
    call("kd_attention_varlen", q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
         out.data_ptr(), out.stride(0), _ptr(gate), gate.stride(0) if gate is not None else 0, cu_q.data_ptr(),
         cu_k.data_ptr(), cu_q.numel() - 1, int(max_q), tq, k.shape[0], hq, k.shape[1], d, float(scale), int(window[0]),
         int(window[1]), status_word(q.device).data_ptr(), sched.data_ptr(), _stream(q))
    return out


def marker_norm(h: torch.Tensor, markers: torch.Tensor, weight: torch.Tensor, mode: int, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``norm(h[markers])`` (M, hidden)."""
    _require(h.is_contiguous(), "h must be contiguous")
    _require(markers.dtype == torch.int64 and markers.is_contiguous(), "markers must be contiguous int64")
    m = markers.numel()
    if out is None:
        out = torch.empty(m, h.shape[1], dtype=torch.bfloat16, device=h.device)
    call("kd_marker_norm", h.data_ptr(), h.shape[1], markers.data_ptr(), m, _ptr(weight), mode, float(eps),
         out.data_ptr(), _stream(h))
    return out


def readout(hidden: torch.Tensor, weight: torch.Tensor, cap: float | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """float32 ``hidden @ weight.T`` (weight float32 (codes, hidden)), soft-capped when ``cap``."""
    _require(hidden.is_contiguous() and weight.is_contiguous() and weight.dtype == torch.float32,
             "readout: contiguous hidden and float32 weight")
    m, codes = hidden.shape[0], weight.shape[0]
    if out is None:
        out = torch.empty(m, codes, dtype=torch.float32, device=hidden.device)
    call("kd_readout", hidden.data_ptr(), m, hidden.shape[1], weight.data_ptr(), codes, float(cap or 0.0),
         out.data_ptr(), _stream(hidden))
    return out


def rope_gather(seqpos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: torch.Tensor | None = None
                ) -> torch.Tensor:
    """The pack's rotary factors for ``qkv_projection``: int32 (rot / 2, T) of packed bf16 (cos, sin) pairs. A position
    past the tables' rows (``cos.shape[0]``) reads as the identity rotation; callers size the tables to the pack."""
    _require(seqpos.dtype == torch.int64 and seqpos.is_contiguous(), "seqpos must be contiguous int64")
    t, rot = seqpos.numel(), cos.shape[1]
    if out is None:
        out = torch.empty(rot // 2, t, dtype=torch.int32, device=seqpos.device)
    call("kd_rope_gather", seqpos.data_ptr(), t, cos.data_ptr(), sin.data_ptr(), cos.shape[0], rot, out.data_ptr(),
         _stream(cos))
    return out


def qkv_projection(a: torch.Tensor, w: torch.Tensor, seqpos: torch.Tensor, heads: int, kv_heads: int,
                   head_dim: int, gated: bool, q_norm: torch.Tensor | None, k_norm: torch.Tensor | None, qk_mode: int,
                   v_mode: int, eps: float, cs: torch.Tensor, rot: int, out: tuple | None = None,
                   scale_a: torch.Tensor | None = None, scale_w: torch.Tensor | None = None) -> tuple:
    """The QKV projection with q/k norms, RoPE and the v norm in its epilogue: (q, k, v, gate or None). bf16 ``a`` and
    ``w``, or e4m3 with per-row scales ``scale_a`` / ``scale_w``; ``cs`` from ``rope_gather`` over the same rows."""
    _rowmajor(a, "a")
    _rowmajor(w, "w")
    _require(seqpos.dtype == torch.int64 and seqpos.is_contiguous(), "seqpos must be contiguous int64")
    t, dev = a.shape[0], a.device
    _require(cs.dtype == torch.int32 and cs.is_contiguous() and cs.shape == (rot // 2, t), "cs: (rot / 2, rows)")
    if out is None:
        q = torch.empty(t, heads, head_dim, dtype=torch.bfloat16, device=dev)
        k = torch.empty(t, kv_heads, head_dim, dtype=torch.bfloat16, device=dev)
        v = torch.empty(t, kv_heads, head_dim, dtype=torch.bfloat16, device=dev)
        gate = torch.empty(t, heads * head_dim, dtype=torch.bfloat16, device=dev) if gated else None
    else:
        q, k, v, gate = out
    tail = (seqpos.data_ptr(), heads, kv_heads, head_dim, int(gated), _ptr(q_norm), _ptr(k_norm), qk_mode, v_mode,
            float(eps), cs.data_ptr(), rot, q.data_ptr(), k.data_ptr(), v.data_ptr(), _ptr(gate),
            status_word(dev).data_ptr(), _stream(a))
    if scale_a is None:
        _require(a.dtype == torch.bfloat16 and w.dtype == torch.bfloat16, "bf16 operands")
        call("kd_qkv_projection", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), t, w.shape[0], a.shape[1],
             *tail)
    else:
        _require(a.dtype == torch.float8_e4m3fn and w.dtype == torch.float8_e4m3fn, "e4m3 operands")
        call("kd_qkv_projection_fp8", a.data_ptr(), a.stride(0), scale_a.data_ptr(), w.data_ptr(), w.stride(0),
             scale_w.data_ptr(), t, w.shape[0], a.shape[1], *tail)
    return q, k, v, gate


def scatter_rows(src: torch.Tensor, rows: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    """``dst[rows] = src`` for bf16 rows (distinct ``rows``, int64 on the device); returns ``dst``."""
    _require(src.dtype == torch.bfloat16 and dst.dtype == torch.bfloat16, "scatter_rows: bf16 rows")
    _require(src.stride(-1) == 1 and dst.stride(-1) == 1, "scatter_rows: rows with unit inner stride")
    _require(rows.dtype == torch.int64 and rows.is_contiguous(), "scatter_rows: contiguous int64 rows")
    width = int(np.prod(src.shape[1:])) if src.dim() > 1 else 1
    _require(width == int(np.prod(dst.shape[1:])), "scatter_rows: row widths differ")
    call("kd_scatter_rows", src.data_ptr(), src.stride(0), rows.data_ptr(), rows.numel(), width, dst.data_ptr(),
         dst.stride(0), _stream(src))
    return dst


def gather_rows(src: torch.Tensor, rows: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``src[rows]`` for bf16 rows (src (T, ...) with contiguous rows; rows int64 on the device)."""
    _require(src.dtype == torch.bfloat16 and src.is_contiguous(), "gather_rows: contiguous bf16 source")
    _require(rows.dtype == torch.int64 and rows.is_contiguous(), "gather_rows: contiguous int64 rows")
    width = src[0].numel() if src.shape[0] else int(np.prod(src.shape[1:]))
    n = rows.numel()
    if out is None:
        out = torch.empty((n, *src.shape[1:]), dtype=src.dtype, device=src.device)
    call("kd_gather_rows", src.data_ptr(), width, rows.data_ptr(), n, width, out.data_ptr(), width, _stream(src))
    return out


# ------------------------------------------------------------------------------------------------ Gated DeltaNet


def conv_silu(x: torch.Tensor, weight: torch.Tensor, seqpos: torch.Tensor, channels: int | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(causal depthwise convolution) of the first ``channels`` columns of bf16 rows ``x`` with taps ``weight``
    (C, K), cut at sequence starts (``seqpos``)."""
    _require(x.dtype == torch.bfloat16 and x.stride(-1) == 1, "conv_silu: bf16 rows")
    _require(weight.dtype == torch.bfloat16 and weight.is_contiguous(), "conv_silu: contiguous bf16 taps")
    _require(seqpos.dtype == torch.int64 and seqpos.is_contiguous(), "seqpos must be contiguous int64")
    t = x.shape[0]
    c = channels if channels is not None else weight.shape[0]
    if out is None:
        out = torch.empty(t, c, dtype=torch.bfloat16, device=x.device)
    call("kd_conv_silu", x.data_ptr(), x.stride(0), t, c, weight.data_ptr(), weight.shape[1], seqpos.data_ptr(),
         out.data_ptr(), out.stride(0), _stream(x))
    return out


def gated_delta_rule(qkv: torch.Tensor, ab: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor,
                     cu: torch.Tensor, k_heads: int, v_heads: int, k_dim: int, v_dim: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """(T, Hv * dv) bf16: the gated delta rule over the packed sequences ``cu`` (int32 on the device); dk = dv = 128
    runs the chunked tensor-core form, which reports a timed-out wait in the device's status word."""
    _require(qkv.dtype == torch.bfloat16 and qkv.stride(-1) == 1, "gated_delta_rule: bf16 qkv rows")
    _require(ab.dtype == torch.bfloat16 and ab.stride(-1) == 1, "gated_delta_rule: bf16 [b | a] rows")
    _require(cu.dtype == torch.int32 and cu.is_contiguous(), "cu: contiguous int32")
    t = qkv.shape[0]
    if out is None:
        out = torch.empty(t, v_heads * v_dim, dtype=torch.bfloat16, device=qkv.device)
    call("kd_gated_delta_rule", qkv.data_ptr(), qkv.stride(0), ab.data_ptr(), ab.stride(0), a_log.data_ptr(),
         dt_bias.data_ptr(), cu.data_ptr(), cu.numel() - 1, t, k_heads, v_heads, k_dim, v_dim, out.data_ptr(),
         out.stride(0), status_word(qkv.device).data_ptr(), _stream(qkv))
    return out


def gated_norm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, heads: int, head_dim: int, eps: float,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3_5RMSNormGated per (row, head): bf16(bf16(w * bf16(norm(x))) * silu(z))."""
    _require(x.dtype == torch.bfloat16 and z.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16,
             "gated_norm: bf16 operands")
    t = x.shape[0]
    if out is None:
        out = torch.empty(t, heads * head_dim, dtype=torch.bfloat16, device=x.device)
    call("kd_gated_norm", x.data_ptr(), x.stride(0), z.data_ptr(), z.stride(0), weight.data_ptr(), t, heads,
         head_dim, float(eps), out.data_ptr(), out.stride(0), _stream(x))
    return out
