"""Tensor-level wrappers over the C ABI (``_lib``): shape and dtype checks, output allocation by PyTorch, the current
stream. Each op is one entry point of libkd_b200; none has a fallback.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import EPI_GEGLU, EPI_RESIDUAL, EPI_STORE, EPI_SWIGLU, NORM_NONE, NORM_ONE_PLUS, NORM_WEIGHT, call

__all__ = ["EPI_GEGLU", "EPI_RESIDUAL", "EPI_STORE", "EPI_SWIGLU", "NORM_NONE", "NORM_ONE_PLUS", "NORM_WEIGHT",
           "add_rmsnorm", "attention_varlen", "check_status", "embed", "gemm", "gemm_fp8", "marker_norm",
           "norm_add", "qkv_norm_rope", "quantize_rows_e4m3", "readout", "rmsnorm", "rmsnorm_e4m3", "rope_table",
           "status_word"]

_STATUS: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The device's int32 status word that pipelined kernels write a timeout into (zero while healthy)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if index not in _STATUS:
        _STATUS[index] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
    return _STATUS[index]


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
