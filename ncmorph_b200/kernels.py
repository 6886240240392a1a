"""Device-backed mirror of ncmorph's ``packages/kernels`` linear entry points.

The host-slice functions keep the reference's Zig signatures and calling
convention (f32 slices carrying bf16 values, caller-owned output written in
place, dimensions passed explicitly) so a caller of
``kernels.matmul_bf16(input, weights, output, token_count, input_width,
output_width)`` (packages/kernels/root.zig:96) can switch by changing the
import. They run on the tcgen05 GEMM in libncm_cuda.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .device import context, need, ptr, stream_of


def _host_f32(a: np.ndarray, n: int, name: str) -> np.ndarray:
    if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags.c_contiguous:
        raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
    if a.size != n:
        raise ValueError(f"{name} has {a.size} elements, expected {n}")
    return a


def _vp(a: np.ndarray | None) -> ctypes.c_void_p | None:
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def matmul_bf16(input: np.ndarray, weights: np.ndarray, output: np.ndarray, token_count: int, input_width: int,
                output_width: int, device: int = 0) -> None:
    """output[T, out] = bf16(input[T, in] . weights[out, in]^T)
    (packages/kernels/root.zig:96-98)."""
    matmul_bf16_bias(input, weights, None, output, token_count, input_width, output_width, device)


def matmul_bf16_bias(input: np.ndarray, weights: np.ndarray, bias: np.ndarray | None, output: np.ndarray,
                     token_count: int, input_width: int, output_width: int, device: int = 0) -> None:
    """BF16 F.linear with an optional bias added to the f32 accumulator before
    the single bf16 rounding (packages/kernels/root.zig:102-104)."""
    _host_f32(input, token_count * input_width, "input")
    _host_f32(weights, output_width * input_width, "weights")
    _host_f32(output, token_count * output_width, "output")
    if bias is not None:
        _host_f32(bias, output_width, "bias")
    _lib.call("ncm_linear_bf16_host_f32", context(device), _vp(input), _vp(weights), _vp(bias), _vp(output),
              token_count, input_width, output_width)


def matmul(input: np.ndarray, weights: np.ndarray, output: np.ndarray, token_count: int, input_width: int,
           output_width: int, device: int = 0) -> None:
    """Stand-in for the f32 kernels.matmul (packages/kernels/root.zig:25-65).
    Computed on the bf16 tensor-core path (operands rounded to bf16, f32
    accumulation, f32 result)."""
    _host_f32(input, token_count * input_width, "input")
    _host_f32(weights, output_width * input_width, "weights")
    _host_f32(output, token_count * output_width, "output")
    _lib.call("ncm_matmul_host_f32", context(device), _vp(input), _vp(weights), _vp(output), token_count,
              input_width, output_width)


def linear_bf16(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Device form: y[M, N] = bf16(x[M, K] . w[N, K]^T + bias[N])."""
    M, K = x.shape
    N = w.shape[0]
    need(x, torch.bfloat16, "x")
    need(w, torch.bfloat16, "w", (N, K))
    if bias is not None:
        need(bias, torch.bfloat16, "bias", (N,))
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    need(out, torch.bfloat16, "out", (M, N))
    _lib.call("ncm_linear_bf16", context(x.device), ptr(x), ptr(w), ptr(bias), ptr(out), M, K, N, stream_of(x))
    return out


def round_bf16(x: torch.Tensor) -> torch.Tensor:
    """bf16 narrowing on the device with the reference rule (RNE, NaN -> 0x7FC0)."""
    need(x, torch.float32, "x")
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.call("ncm_f32_to_bf16", context(x.device), ptr(x), ptr(out), x.numel(), stream_of(x))
    return out


def widen_bf16(x: torch.Tensor) -> torch.Tensor:
    """Exact bf16 -> f32 widening on the device."""
    need(x, torch.bfloat16, "x")
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    _lib.call("ncm_bf16_to_f32", context(x.device), ptr(x), ptr(out), x.numel(), stream_of(x))
    return out
