"""The quantiser's pieces around the RVQ levels on B200
(research/reference/vq_forward_semantics.md): pre-quantisation GroupNorm
(:43-49), the learned level-0 down/up cascade of stride-4 convolutions
(:127-139) and the codebook EMA update (:141-173). The convolutions run as
tcgen05 GEMMs; the EMA statistics are deterministic (rows summed per code in
row order)."""
from __future__ import annotations

import torch

from . import _lib
from .device import context, need, ptr, stream_of

bf16 = torch.bfloat16


def group_norm(x: torch.Tensor, groups: int, eps: float = 1e-5) -> torch.Tensor:
    """GroupNorm(groups, C, affine=False) over x [B, T, C] f32 (channels last)."""
    B, T, C = x.shape
    need(x, torch.float32, "x")
    y = torch.empty_like(x)
    _lib.call("ncm_group_norm", context(x.device), ptr(x), ptr(y), B, T, C, groups, float(eps), stream_of(x))
    return y


def conv_down4(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """Conv1d(C, C, kernel 4, stride 4) along time: x [B, L, C] bf16 -> [B, L/4, C]; weight [C, C, 4]."""
    B, L, C = x.shape
    need(x, bf16, "x")
    need(weight, bf16, "weight", (C, C, 4))
    if bias is not None:
        need(bias, bf16, "bias", (C,))
    y = torch.empty((B, L // 4, C), dtype=bf16, device=x.device)
    _lib.call("ncm_conv_down4", context(x.device), ptr(x), ptr(weight), ptr(bias), ptr(y), B, L, C, stream_of(x))
    return y


def conv_up4(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """ConvTranspose1d(C, C, kernel 4, stride 4): x [B, L, C] bf16 -> [B, 4L, C]; weight [C_in, C_out, 4]."""
    B, L, C = x.shape
    need(x, bf16, "x")
    need(weight, bf16, "weight", (C, C, 4))
    if bias is not None:
        need(bias, bf16, "bias", (C,))
    y = torch.empty((B, 4 * L, C), dtype=bf16, device=x.device)
    _lib.call("ncm_conv_up4", context(x.device), ptr(x), ptr(weight), ptr(bias), ptr(y), B, L, C, stream_of(x))
    return y


def level0_down(x: torch.Tensor, weights, biases) -> torch.Tensor:
    """The learned level-0 down-sampler: the cascade of stride-4 Conv1d stages (1024 -> 1 positions for five)."""
    for w, b in zip(weights, biases):
        x = conv_down4(x, w, b)
    return x


def level0_up(x: torch.Tensor, weights, biases) -> torch.Tensor:
    """The learned level-0 up-sampler: the cascade of stride-4 ConvTranspose1d stages."""
    for w, b in zip(weights, biases):
        x = conv_up4(x, w, b)
    return x


class CodebookEMA:
    """EMA buffers of one level (N_k zeros, m_k a copy of the initial
    codebook, decay 0.99, eps 1e-5 as the released configuration) and the
    update after each training forward. With a torch.distributed process
    group the per-code counts and sums are all-reduced before the update, as
    the upstream quantiser does under data parallelism."""

    def __init__(self, codebook: torch.Tensor, decay: float = 0.99, eps: float = 1e-5):
        K, D = codebook.shape
        self.decay, self.eps = float(decay), float(eps)
        self.count = torch.zeros(K, dtype=torch.float32, device=codebook.device)
        self.sum = codebook.float().contiguous().clone()
        self.K, self.D = K, D

    def stats(self, u: torch.Tensor, codes: torch.Tensor):
        """(counts [K], sums [K, D]) of this batch's rows u [N, D] f32 by code."""
        N, D = u.shape
        need(u, torch.float32, "u")
        need(codes, torch.int32, "codes", (N,))
        counts = torch.empty(self.K, dtype=torch.float32, device=u.device)
        sums = torch.empty((self.K, self.D), dtype=torch.float32, device=u.device)
        _lib.call("ncm_ema_code_stats", context(u.device), ptr(u), ptr(codes), ptr(counts), ptr(sums), N, D, self.K,
                  stream_of(u))
        return counts, sums

    def update(self, u: torch.Tensor, codes: torch.Tensor, codebook_bf16: torch.Tensor | None = None,
               codebook_f32: torch.Tensor | None = None, group=None) -> None:
        counts, sums = self.stats(u, codes)
        if group is not None or (torch.distributed.is_available() and torch.distributed.is_initialized()):
            torch.distributed.all_reduce(counts, group=group)
            torch.distributed.all_reduce(sums, group=group)
        for t, dt, name in ((codebook_bf16, bf16, "codebook_bf16"), (codebook_f32, torch.float32, "codebook_f32")):
            if t is not None:
                need(t, dt, name, (self.K, self.D))
        _lib.call("ncm_ema_update", context(u.device), ptr(counts), ptr(sums), ptr(self.count), ptr(self.sum),
                  ptr(codebook_f32), ptr(codebook_bf16), self.K, self.D, self.decay, self.eps, stream_of(u))
