"""Per-device library contexts and argument plumbing for torch tensors.

PyTorch is used here only for device memory and streams: tensors are passed
to the C ABI as raw device pointers together with torch's current stream.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_contexts: dict[int, ctypes.c_void_p] = {}
_lock = threading.Lock()


def context(device: int | torch.device | None = None) -> ctypes.c_void_p:
    """Returns (creating once) the library context of a CUDA device."""
    if device is None:
        device = torch.cuda.current_device()
    if isinstance(device, torch.device):
        device = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        ctx = _contexts.get(device)
        if ctx is None:
            ctx = ctypes.c_void_p()
            _lib.call("ncm_ctx_create", int(device), ctypes.byref(ctx))
            _contexts[device] = ctx
        return ctx


def release_all() -> None:
    """Destroys every context (the library frees its workspaces)."""
    with _lock:
        for ctx in _contexts.values():
            _lib.load().ncm_ctx_destroy(ctx)
        _contexts.clear()


def stream_of(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def need(t: torch.Tensor, dtype: torch.dtype, name: str, shape: tuple | None = None) -> torch.Tensor:
    """Validates a device tensor argument (dtype, contiguity, shape)."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    return t


def sync(device: int | torch.device | None = None) -> None:
    """Waits for torch's current stream and reports device-side failures."""
    dev = torch.device("cuda", device) if isinstance(device, int) else (device or torch.device("cuda"))
    _lib.call("ncm_sync", context(dev), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
