"""Device mirror of ncmorph's NCM body forward (src/ncm_model.zig:77-250) in
bf16 (the layer of src/decoder.zig:168-216), plus the per-op entry points it
is built from: RMSNorm, embedding gather, RoPE tables and masked attention.

Masks: "causal" (kernels.causal_mask), "block_diagonal" (ncm_mask.zig:10-42,
ncmorph's only NCM mask) and "block_causal" (each level also attends to
every earlier level; the BASELINE config-4 pattern).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from .device import context, need, ptr, stream_of

MASK_MODES = {"causal": 0, "block_diagonal": 1, "block_causal": 2}
bf16 = torch.bfloat16


def make_mask(mode: str, prefix_length: int = 0, level_lengths=(), prefix_pad=(),
              sliding_window: int | None = None) -> _lib.Mask:
    m = _lib.Mask()
    m.mode = MASK_MODES[mode]
    m.sliding_window = int(sliding_window or 0)
    m.prefix_length = int(prefix_length)
    bits = 0
    for i, padded in enumerate(prefix_pad):
        if padded:
            bits |= 1 << i
    m.prefix_pad_mask = bits
    m.num_levels = len(level_lengths)
    for i, n in enumerate(level_lengths):
        m.level_lengths[i] = int(n)
    return m


def level_positions(prefix_length: int, level_lengths) -> np.ndarray:
    """ncm_position.fill_level_positions (src/ncm_position.zig:11-22)."""
    pos = list(range(prefix_length))
    for n in level_lengths:
        pos.extend(range(n))
    return np.asarray(pos, dtype=np.int32)


def rope_tables(head_dim: int, theta: float, positions, llama3: tuple | None = None
                ) -> tuple[np.ndarray, np.ndarray]:
    """Host RoPE tables [T, head_dim] with libm, as the reference builds them:
    rope_default's frequencies, or rope_llama3's when `llama3` = (factor,
    low_freq_factor, high_freq_factor, original_max_position_embeddings)."""
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    T = pos.size
    c = np.empty((T, head_dim), np.float32)
    s = np.empty((T, head_dim), np.float32)
    vp = ctypes.c_void_p
    if llama3 is None:
        _lib.call("ncm_rope_tables_host", head_dim, float(theta), vp(pos.ctypes.data), T, vp(c.ctypes.data),
                  vp(s.ctypes.data))
    else:
        factor, low, high, orig = llama3
        _lib.call("ncm_rope_tables_llama3_host", head_dim, float(theta), float(factor), float(low), float(high),
                  int(orig), vp(pos.ctypes.data), T, vp(c.ctypes.data), vp(s.ctypes.data))
    return c, s


def rms_norm_bf16(x: torch.Tensor, weight: torch.Tensor, eps: float, bias: torch.Tensor | None = None):
    rows, width = x.shape
    need(x, bf16, "x")
    need(weight, bf16, "weight", (width,))
    y = torch.empty_like(x)
    _lib.call("ncm_rms_norm_bf16", context(x.device), ptr(x), ptr(weight), ptr(bias), ptr(y), rows, width,
              float(eps), stream_of(x))
    return y


def embedding_gather(table: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    vocab, width = table.shape
    need(table, bf16, "table")
    need(ids, torch.int32, "ids")
    out = torch.empty((ids.numel(), width), dtype=bf16, device=table.device)
    _lib.call("ncm_embedding_gather", context(table.device), ptr(table), vocab, width, ptr(ids), ids.numel(),
              ptr(out), stream_of(table))
    return out


def attention_bf16(qkv: torch.Tensor, heads: int, kv_heads: int, mask: _lib.Mask,
                   cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                   q_norm: torch.Tensor | None = None, k_norm: torch.Tensor | None = None,
                   eps: float = 1e-6) -> torch.Tensor:
    """Context [T, heads*64] from fused QKV rows [T, (heads + 2*kv_heads)*64];
    QK-norm (if q_norm/k_norm [64] bf16 are given, with eps) and then RoPE (if
    cos/sin given) are applied to qkv in place."""
    T, stride = qkv.shape
    need(qkv, bf16, "qkv")
    out = torch.empty((T, heads * 64), dtype=bf16, device=qkv.device)
    if q_norm is None and k_norm is None:
        _lib.call("ncm_attention_bf16", context(qkv.device), ptr(qkv), stride, ptr(cos), ptr(sin), ptr(out), T, heads,
                  kv_heads, ctypes.byref(mask), stream_of(qkv))
    else:
        _lib.call("ncm_attention_qk_norm_bf16", context(qkv.device), ptr(qkv), stride, ptr(cos), ptr(sin),
                  ptr(q_norm), ptr(k_norm), eps, ptr(out), T, heads, kv_heads, ctypes.byref(mask), stream_of(qkv))
    return out


@dataclass
class LayerWeights:
    ln_1: torch.Tensor
    qkv: torch.Tensor
    o: torch.Tensor
    ln_2: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    qkv_bias: torch.Tensor | None = None
    o_bias: torch.Tensor | None = None
    # QK-norm scales [64] bf16 (ncm_model.zig:42-43): both or None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None


@dataclass
class Weights:
    input_projection: torch.Tensor
    input_projection_bias: torch.Tensor
    level_embedding: torch.Tensor
    final_norm: torch.Tensor
    layers: list = field(default_factory=list)
    final_norm_bias: torch.Tensor | None = None
    # post_upsample_convs (ncm_model.zig:71): [levels, vq, vq, 3] bf16 and [levels, vq] f32
    post_conv_weight: torch.Tensor | None = None
    post_conv_bias: torch.Tensor | None = None


@dataclass
class Config:
    hidden_size: int
    vq_width: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    level_lengths: tuple
    prefix_length: int = 0
    # "causal" is ncm_model's source_causal (src/ncm_model.zig:199-203), which
    # may carry a sliding window; the block masks take none
    mask: str = "block_causal"
    sliding_window: int | None = None
    rms_norm_epsilon: float = 1e-5
    rope_theta: float = 500000.0
    use_level_encoding: bool = True
    head_dim: int = 64
    # Llama 3 frequency scaling (rope_llama3, packages/kernels/root.zig:636-666):
    # (factor, low_freq_factor, high_freq_factor, original_max_position_embeddings),
    # or None for rope_default
    rope_llama3: tuple | None = None

    @property
    def seq_len(self) -> int:
        return self.prefix_length + sum(self.level_lengths)


def _vp(t):
    return None if t is None else t.data_ptr()


def forward(cfg: Config, w: Weights, inputs: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """ncm_model.forward on the GPU: inputs [T, vq_width] bf16 -> hidden [T, hidden] bf16."""
    T = cfg.seq_len
    need(inputs, bf16, "inputs", (T, cfg.vq_width))
    c = _lib.DecoderConfig()
    c.hidden_size, c.vq_width = cfg.hidden_size, cfg.vq_width
    c.num_attention_heads, c.num_key_value_heads = cfg.num_attention_heads, cfg.num_key_value_heads
    c.head_dim, c.intermediate_size = cfg.head_dim, cfg.intermediate_size
    c.rms_norm_epsilon, c.rope_theta = cfg.rms_norm_epsilon, cfg.rope_theta
    c.use_level_encoding = int(cfg.use_level_encoding)
    c.mask = make_mask(cfg.mask, cfg.prefix_length, cfg.level_lengths, sliding_window=cfg.sliding_window)
    if cfg.rope_llama3 is not None:
        c.rope_type = 1
        (c.rope_factor, c.rope_low_freq_factor, c.rope_high_freq_factor,
         c.rope_original_max_position_embeddings) = cfg.rope_llama3
    layers = (_lib.DecoderLayerWeights * len(w.layers))()
    for i, L in enumerate(w.layers):
        for name in ("ln_1", "qkv", "qkv_bias", "o", "o_bias", "ln_2", "gate_up", "down", "q_norm", "k_norm"):
            setattr(layers[i], name, _vp(getattr(L, name)))
    W = _lib.DecoderWeights()
    W.input_projection = _vp(w.input_projection)
    W.input_projection_bias = _vp(w.input_projection_bias)
    W.level_embedding = _vp(w.level_embedding)
    W.final_norm = _vp(w.final_norm)
    W.final_norm_bias = _vp(w.final_norm_bias)
    W.num_layers = len(w.layers)
    W.layers = layers
    if w.post_conv_weight is not None:
        L, V = len(cfg.level_lengths), cfg.vq_width
        need(w.post_conv_weight, bf16, "post_conv_weight", (L, V, V, 3))
        need(w.post_conv_bias, torch.float32, "post_conv_bias", (L, V))
    W.post_conv_weight = _vp(w.post_conv_weight)
    W.post_conv_bias = _vp(w.post_conv_bias)
    if out is None:
        out = torch.empty((T, cfg.hidden_size), dtype=bf16, device=inputs.device)
    _lib.call("ncm_ncm_forward", context(inputs.device), ctypes.byref(c), ctypes.byref(W), ptr(inputs), ptr(out),
              stream_of(inputs))
    return out


def apply_post_upsample_conv(input: np.ndarray, weight: np.ndarray, bias: np.ndarray, row_count: int, width: int,
                             device: int = 0) -> None:
    """ncm_model.apply_post_upsample_conv (src/ncm_model.zig:296-326) on the GPU:
    input [row_count, width] f32 (host) becomes input + bias + Conv1d_k3(input)
    in place; weight [width, width, 3] and bias [width] are f32 host arrays
    holding bf16 values. The convolution runs on tcgen05 with bf16 operands."""
    for a, n, name in ((input, row_count * width, "input"), (weight, width * width * 3, "weight"),
                       (bias, width, "bias")):
        if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags.c_contiguous:
            raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
        if a.size != n:
            raise ValueError(f"{name} has {a.size} elements, expected {n}")
    _lib.call("ncm_post_upsample_conv_host_f32", context(device), ctypes.c_void_p(input.ctypes.data),
              ctypes.c_void_p(weight.ctypes.data), ctypes.c_void_p(bias.ctypes.data), row_count, width)


def tied_head_logits(z: torch.Tensor, codebook: torch.Tensor, log_inv_T: float = 0.0,
                     bias: torch.Tensor | None = None, esq: torch.Tensor | None = None) -> torch.Tensor:
    """_TiedCodebookHead (PROJECT.md:222): logits [T, K] f32 =
    (2 z.E^T - E_sq) / mean(E_sq) * exp(log_inv_T) + bias, z [T, d] bf16, E [K, d] bf16."""
    T, d = z.shape
    K = codebook.shape[0]
    need(z, bf16, "z")
    need(codebook, bf16, "codebook", (K, d))
    for t, name in ((bias, "bias"), (esq, "esq")):
        if t is not None:
            need(t, torch.float32, name, (K,))
    out = torch.empty((T, K), dtype=torch.float32, device=z.device)
    _lib.call("ncm_tied_head_logits", context(z.device), ptr(z), ptr(codebook), ptr(esq), ptr(bias),
              float(log_inv_T), ptr(out), T, d, K, stream_of(z))
    return out


def tied_head_argmax(z: torch.Tensor, codebook: torch.Tensor, log_inv_T: float = 0.0,
                     bias: torch.Tensor | None = None, esq: torch.Tensor | None = None) -> torch.Tensor:
    """argmax_k of tied_head_logits (lowest k on ties) without materialising the logits -> int32 [T]."""
    T, d = z.shape
    K = codebook.shape[0]
    need(z, bf16, "z")
    need(codebook, bf16, "codebook", (K, d))
    for t, name in ((bias, "bias"), (esq, "esq")):
        if t is not None:
            need(t, torch.float32, name, (K,))
    codes = torch.empty(T, dtype=torch.int32, device=z.device)
    _lib.call("ncm_tied_head_argmax", context(z.device), ptr(z), ptr(codebook), ptr(esq), ptr(bias),
              float(log_inv_T), ptr(codes), T, d, K, stream_of(z))
    return codes
