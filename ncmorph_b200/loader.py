"""Checkpoint tensors straight to the GPU as bf16: the device-side form of
ncmorph's safetensors loading (packages/safetensors/root.zig:148-200
`header_length`/`parse_header`; src/loader.zig:286-345 `read_tensor`).

The header is parsed and validated on the host as the reference does it
(8-byte little-endian length, JSON object, contiguous data offsets that
match each tensor's shape and dtype, file size = 8 + header + data); the
tensor bytes then move file -> pinned staging -> device inside
libncm_cuda.so (ncm_load_tensor_bf16), never widened to f32.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass

import torch

from . import _lib
from .device import context, ptr, stream_of

MAX_HEADER = 100 * 1024 * 1024
DTYPE_CODES = {"BF16": 0, "F16": 1, "F32": 2}
DTYPE_BITS = {"BOOL": 8, "U8": 8, "I8": 8, "U16": 16, "I16": 16, "F16": 16, "BF16": 16, "U32": 32, "I32": 32,
              "F32": 32, "U64": 64, "I64": 64, "F64": 64, "F8_E5M2": 8, "F8_E4M3": 8}


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    data_begin: int
    data_end: int


@dataclass(frozen=True)
class Header:
    header_len: int
    data_len: int
    tensors: dict

    def offset(self, t: TensorInfo) -> int:
        """Absolute file offset of a tensor's first byte."""
        return 8 + self.header_len + t.data_begin


def parse_header(path: str | os.PathLike) -> Header:
    """Reads and validates a safetensors header (the checks of parse_header)."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        prefix = f.read(8)
        if len(prefix) < 8:
            raise ValueError("header too small")
        (n,) = struct.unpack("<Q", prefix)
        if n > MAX_HEADER:
            raise ValueError("header too large")
        raw = f.read(n)
    if len(raw) != n:
        raise ValueError("invalid header length")
    fields = json.loads(raw.decode("utf-8"))
    if not isinstance(fields, dict):
        raise ValueError("invalid header")
    tensors = []
    for name, v in fields.items():
        if name == "__metadata__":
            continue
        dtype, shape, (b, e) = v["dtype"], tuple(int(d) for d in v["shape"]), v["data_offsets"]
        if dtype not in DTYPE_BITS:
            raise ValueError(f"unknown dtype {dtype}")
        tensors.append(TensorInfo(name, dtype, shape, int(b), int(e)))
    tensors.sort(key=lambda t: (t.data_begin, t.data_end))
    at = 0
    for t in tensors:
        if t.data_begin != at or t.data_end < t.data_begin:
            raise ValueError("invalid offsets")
        count = 1
        for d in t.shape:
            count *= d
        bits = count * DTYPE_BITS[t.dtype]
        if bits % 8 or t.data_end - t.data_begin != bits // 8:
            raise ValueError(f"size mismatch for {t.name}")
        at = t.data_end
    if 8 + n + at != size:
        raise ValueError("file size mismatch")
    return Header(n, at, {t.name: t for t in tensors})


def load_tensor_bf16(path: str | os.PathLike, name: str, device=None, header: Header | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One tensor to the device as bf16 (BF16 bit for bit; F16/F32 rounded to nearest even)."""
    h = header if header is not None else parse_header(path)
    t = h.tensors[name]
    if t.dtype not in DTYPE_CODES:
        raise ValueError(f"{name}: dtype {t.dtype} is not BF16, F16 or F32")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty(t.shape, dtype=torch.bfloat16, device=dev)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != t.shape or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous bf16 tensor of shape {t.shape}")
    _lib.call("ncm_load_tensor_bf16", context(out.device), os.fsencode(path), h.offset(t), t.data_end - t.data_begin,
              DTYPE_CODES[t.dtype], ptr(out), stream_of(out))
    return out


def load_all_bf16(path: str | os.PathLike, device=None) -> dict:
    """Every BF16/F16/F32 tensor of one safetensors file, as device bf16 tensors."""
    h = parse_header(path)
    return {n: load_tensor_bf16(path, n, device, h) for n, t in h.tensors.items() if t.dtype in DTYPE_CODES}
