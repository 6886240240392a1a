"""Residual vector quantisation on B200: the device-side mirror of the
multiscale RVQ tokenizer forward that ncmorph specifies for its planned
``packages/vq`` (research/reference/vq_forward_semantics.md:59-82,
research/ncm_facts.md:62-82, PROJECT.md:250-285).

Numerics (fixed by this implementation, restated by the CPU oracle):
  * residuals are f32; the distance GEMM operand is bf16(residual);
  * codebooks are bf16; ||e_k||^2 is summed exactly (f64) and rounded to f32;
  * dist = ||e_k||^2 - 2 * (bf16(r) . e_k) with f32 accumulation on tcgen05;
    ||r||^2 is dropped (constant per row);
  * argmin picks the lowest index among equal distances (torch.argmin rule);
  * the residual update r -= e[code] is exact f32 arithmetic;
  * reconstructions sum the chosen codewords in f32 (level order) and round
    once to bf16.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .device import context, need, ptr, stream_of

bf16 = torch.bfloat16


def code_sqnorm(codebook: torch.Tensor) -> torch.Tensor:
    """||e_k||^2 for a bf16 codebook [..., K, D] -> f32 [..., K] (R1)."""
    need(codebook, bf16, "codebook")
    D = codebook.shape[-1]
    K = codebook.numel() // D
    out = torch.empty(codebook.shape[:-1], dtype=torch.float32, device=codebook.device)
    _lib.call("ncm_code_sqnorm", context(codebook.device), ptr(codebook), ptr(out), K, D, stream_of(codebook))
    return out


def rvq_level(residual: torch.Tensor, codebook: torch.Tensor, sqnorm: torch.Tensor | None = None,
              codes: torch.Tensor | None = None) -> torch.Tensor:
    """One RVQ level (R2+R3): returns int32 codes [N]; updates `residual` in place."""
    N, D = residual.shape
    K = codebook.shape[0]
    need(residual, torch.float32, "residual")
    need(codebook, bf16, "codebook", (K, D))
    if sqnorm is not None:
        need(sqnorm, torch.float32, "sqnorm", (K,))
    if codes is None:
        codes = torch.empty(N, dtype=torch.int32, device=residual.device)
    need(codes, torch.int32, "codes", (N,))
    _lib.call("ncm_rvq_level", context(residual.device), ptr(residual), ptr(codebook), ptr(sqnorm), ptr(codes),
              N, D, K, stream_of(residual))
    return codes


def rvq_level_top2(residual: torch.Tensor, codebook: torch.Tensor, sqnorm: torch.Tensor | None = None):
    """rvq_level that also returns each row's relative top-2 distance gap
    (d2 - d1) / (||bf16(r)||^2 + d1). Returns (codes int32 [N], gap f32 [N])."""
    N, D = residual.shape
    K = codebook.shape[0]
    need(residual, torch.float32, "residual")
    need(codebook, bf16, "codebook", (K, D))
    if sqnorm is not None:
        need(sqnorm, torch.float32, "sqnorm", (K,))
    codes = torch.empty(N, dtype=torch.int32, device=residual.device)
    gap = torch.empty(N, dtype=torch.float32, device=residual.device)
    _lib.call("ncm_rvq_level_top2", context(residual.device), ptr(residual), ptr(codebook), ptr(sqnorm), ptr(codes),
              ptr(gap), N, D, K, stream_of(residual))
    return codes, gap


def rvq_encode(x: torch.Tensor, codebooks: torch.Tensor, sqnorms: torch.Tensor | None = None, *,
               want_recon: bool = True, want_residual: bool = False,
               codes: torch.Tensor | None = None, recon: torch.Tensor | None = None):
    """L residual levels over bf16 x [N, D] with bf16 codebooks [L, K, D].

    Returns (codes int32 [L, N], recon bf16 [N, D] or None, residual f32 [N, D] or None).
    """
    N, D = x.shape
    L, K, D2 = codebooks.shape
    if D2 != D:
        raise ValueError("codebook width differs from x")
    need(x, bf16, "x")
    need(codebooks, bf16, "codebooks")
    if sqnorms is not None:
        need(sqnorms, torch.float32, "sqnorms", (L, K))
    dev = x.device
    if codes is None:
        codes = torch.empty((L, N), dtype=torch.int32, device=dev)
    need(codes, torch.int32, "codes", (L, N))
    if want_recon and recon is None:
        recon = torch.empty((N, D), dtype=bf16, device=dev)
    if recon is not None:
        need(recon, bf16, "recon", (N, D))
    residual = torch.empty((N, D), dtype=torch.float32, device=dev) if want_residual else None
    _lib.call("ncm_rvq_encode", context(dev), ptr(x), ptr(codebooks), ptr(sqnorms), L, ptr(codes), ptr(recon),
              ptr(residual), N, D, K, stream_of(x))
    return codes, recon, residual


def rvq_encode_host(x_host: torch.Tensor, codebooks: torch.Tensor, sqnorms: torch.Tensor | None = None, *,
                    codes_host: torch.Tensor | None = None, recon_host: torch.Tensor | None = None,
                    want_recon: bool = True):
    """Host-buffer encode: x_host [N, D] bf16 in host memory (pin it for full
    copy speed), codebooks [L, K, D] on the device. Copies and compute are
    pipelined in row chunks inside the library; returns host tensors
    (codes [L, N] int32, recon [N, D] bf16 or None) once they are filled."""
    if x_host.is_cuda or not x_host.is_contiguous() or x_host.dtype != bf16:
        raise ValueError("x_host must be a contiguous bf16 CPU tensor")
    N, D = x_host.shape
    L, K, D2 = codebooks.shape
    if D2 != D:
        raise ValueError("codebook width differs from x")
    need(codebooks, bf16, "codebooks")
    if sqnorms is not None:
        need(sqnorms, torch.float32, "sqnorms", (L, K))
    if codes_host is None:
        codes_host = torch.empty((L, N), dtype=torch.int32, pin_memory=x_host.is_pinned())
    if want_recon and recon_host is None:
        recon_host = torch.empty((N, D), dtype=bf16, pin_memory=x_host.is_pinned())
    for t, name in ((codes_host, "codes_host"), (recon_host, "recon_host")):
        if t is not None and (t.is_cuda or not t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous CPU tensor")
    dev = codebooks.device
    _lib.call("ncm_rvq_encode_host", context(dev), ptr(x_host), ptr(codebooks), ptr(sqnorms), L, ptr(codes_host),
              ptr(recon_host), N, D, K, stream_of(codebooks))
    return codes_host, recon_host


def rvq_decode(codes: torch.Tensor, codebooks: torch.Tensor, recon: torch.Tensor | None = None) -> torch.Tensor:
    """recon[n] = bf16(sum_l e_l[codes[l, n]]) (R5). A row holding an
    out-of-range code is left unwritten and the context reports NCM_ERANGE."""
    L, N = codes.shape
    L2, K, D = codebooks.shape
    if L2 != L:
        raise ValueError("codes and codebooks disagree on the number of levels")
    need(codes, torch.int32, "codes")
    need(codebooks, bf16, "codebooks")
    if recon is None:
        recon = torch.empty((N, D), dtype=bf16, device=codes.device)
    need(recon, bf16, "recon", (N, D))
    _lib.call("ncm_rvq_decode", context(codes.device), ptr(codes), ptr(codebooks), L, ptr(recon), N, D, K,
              stream_of(codes))
    return recon


def pool_avg(x: torch.Tensor, factor: int) -> torch.Tensor:
    """Area pooling [B, T, D] -> [B, T/factor, D] in f32 (R4)."""
    B, T, D = x.shape
    need(x, torch.float32, "x")
    y = torch.empty((B, T // factor, D), dtype=torch.float32, device=x.device)
    _lib.call("ncm_pool_avg", context(x.device), ptr(x), ptr(y), B, T, D, int(factor), stream_of(x))
    return y


UPSAMPLE_MODES = {"nearest": 0, "linear": 1}


def upsample(q: torch.Tensor, out_len: int, mode: str = "linear") -> torch.Tensor:
    """F.interpolate(size=out_len) along time of q [B, Tq, D] f32 (the
    quantiser's U_i, vq_forward_semantics.md:82): nearest or linear
    (align_corners=False). Returns f32 [B, out_len, D]."""
    B, Tq, D = q.shape
    need(q, torch.float32, "q")
    out = torch.empty((B, out_len, D), dtype=torch.float32, device=q.device)
    _lib.call("ncm_upsample", context(q.device), ptr(q), ptr(out), B, Tq, out_len, D, UPSAMPLE_MODES[mode],
              stream_of(q))
    return out


def conv1d_k3(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
              segments: list[int] | None = None, alpha: float = 1.0, beta: float = 1.0,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """out = alpha * x + beta * (bias + Conv1d(x; weight, kernel 3, padding 1))
    along the rows of x [rows, width] f32, each segment zero-padded on its own.
    weight [width, width, 3] bf16 (the Conv1d layout). alpha = beta = 1 is
    ncm_model.apply_post_upsample_conv; alpha = 1 - r, beta = r is Phi."""
    rows, width = x.shape
    need(x, torch.float32, "x")
    need(weight, bf16, "weight", (width, width, 3))
    if bias is not None:
        need(bias, torch.float32, "bias", (width,))
    if out is None:
        out = torch.empty_like(x)
    need(out, torch.float32, "out", (rows, width))
    lens = None
    nseg = 1
    if segments is not None:
        nseg = len(segments)
        lens = (ctypes.c_int64 * nseg)(*[int(n) for n in segments])
    _lib.call("ncm_conv1d_k3", context(x.device), ptr(x), ptr(weight), ptr(bias), ptr(out), rows, width, nseg, lens,
              float(alpha), float(beta), stream_of(x))
    return out


def tokenizer_config(batch: int, seq_len: int, model_width: int, vq_width: int, codebook_size: int,
                     pool_factors: list[int], levels_per_scale: int, upsample: str = "nearest",
                     phi_ratio: float = 0.5) -> _lib.TokenizerConfig:
    cfg = _lib.TokenizerConfig()
    cfg.batch, cfg.seq_len, cfg.model_width, cfg.vq_width = batch, seq_len, model_width, vq_width
    cfg.codebook_size = codebook_size
    cfg.num_scales = len(pool_factors)
    cfg.levels_per_scale = levels_per_scale
    for i, f in enumerate(pool_factors):
        cfg.pool_factors[i] = int(f)
    cfg.upsample_mode = UPSAMPLE_MODES[upsample]
    cfg.phi_ratio = float(phi_ratio)
    return cfg


def _check_phi(phi_weight, phi_bias, S, D):
    if (phi_weight is None) != (phi_bias is None):
        raise ValueError("pass both phi_weight and phi_bias, or neither")
    if phi_weight is not None:
        need(phi_weight, bf16, "phi_weight", (S, D, D, 3))
        need(phi_bias, torch.float32, "phi_bias", (S, D))


def _split_codes(codes_flat, L, rows):
    codes, off = [], 0
    for r in rows:
        codes.append(codes_flat[off:off + L * r].view(L, r))
        off += L * r
    return codes


def tokenizer_forward(x: torch.Tensor, w_in: torch.Tensor, codebooks: torch.Tensor, w_out: torch.Tensor,
                      pool_factors: list[int], *, b_in: torch.Tensor | None = None,
                      b_out: torch.Tensor | None = None, sqnorms: torch.Tensor | None = None,
                      upsample: str = "nearest", phi_weight: torch.Tensor | None = None,
                      phi_bias: torch.Tensor | None = None, phi_ratio: float = 0.5):
    """Multiscale RVQ tokenizer forward (R6).

    x [B, T, Din] bf16; w_in [D, Din]; codebooks [S, L, K, D]; w_out [Din, D].
    upsample: "nearest" (default) or "linear"; phi_weight [S, D, D, 3] bf16 and
    phi_bias [S, D] f32 add the quantiser's Phi after each scale's upsampling.
    Returns (codes: list over scales of int32 [L, B*T/f_s], recon bf16 [B, T, D], y bf16 [B, T, Din]).
    """
    B, T, Din = x.shape
    S, L, K, D = codebooks.shape
    if len(pool_factors) != S:
        raise ValueError("one pool factor per scale is required")
    need(x, bf16, "x")
    need(w_in, bf16, "w_in", (D, Din))
    need(codebooks, bf16, "codebooks")
    need(w_out, bf16, "w_out", (Din, D))
    if sqnorms is not None:
        need(sqnorms, torch.float32, "sqnorms", (S, L, K))
    _check_phi(phi_weight, phi_bias, S, D)
    dev = x.device
    rows = [B * T // f for f in pool_factors]
    codes_flat = torch.empty(sum(L * r for r in rows), dtype=torch.int32, device=dev)
    recon = torch.empty((B, T, D), dtype=bf16, device=dev)
    y = torch.empty((B, T, Din), dtype=bf16, device=dev)
    cfg = tokenizer_config(B, T, Din, D, K, pool_factors, L, upsample, phi_ratio)
    _lib.call("ncm_tokenizer_forward_ex", context(dev), ctypes.byref(cfg), ptr(x), ptr(w_in), ptr(b_in),
              ptr(codebooks), ptr(sqnorms), ptr(phi_weight), ptr(phi_bias), ptr(w_out), ptr(b_out),
              ptr(codes_flat), ptr(recon), ptr(y), stream_of(x))
    return _split_codes(codes_flat, L, rows), recon, y


def multiscale_decode(codes: list[torch.Tensor], codebooks: torch.Tensor, batch: int, seq_len: int,
                      pool_factors: list[int], *, upsample: str = "nearest", phi_weight: torch.Tensor | None = None,
                      phi_bias: torch.Tensor | None = None, phi_ratio: float = 0.5) -> torch.Tensor:
    """recon [B, T, D] bf16 = bf16(sum_s Phi_s(up(q_s))) from per-scale codes
    [L, B*T/f_s] as tokenizer_forward returns them (R5 at every scale)."""
    S, L, K, D = codebooks.shape
    if len(pool_factors) != S or len(codes) != S:
        raise ValueError("one pool factor and one code tensor per scale are required")
    need(codebooks, bf16, "codebooks")
    _check_phi(phi_weight, phi_bias, S, D)
    for s, c in enumerate(codes):
        need(c, torch.int32, f"codes[{s}]", (L, batch * seq_len // pool_factors[s]))
    dev = codebooks.device
    flat = torch.cat([c.reshape(-1) for c in codes])
    recon = torch.empty((batch, seq_len, D), dtype=bf16, device=dev)
    cfg = tokenizer_config(batch, seq_len, 0, D, K, pool_factors, L, upsample, phi_ratio)
    _lib.call("ncm_multiscale_decode", context(dev), ctypes.byref(cfg), ptr(flat), ptr(codebooks), ptr(phi_weight),
              ptr(phi_bias), ptr(recon), stream_of(codebooks))
    return recon
