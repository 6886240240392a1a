"""ctypes binding of the CPU oracle (oracle/build/libncm_oracle.so).

TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, where it is the checker or the timed CPU
baseline — never by the ncmorph_b200 package.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB = HERE / "build" / "libncm_oracle.so"

_lib = None
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
szp = np.ctypeslib.ndpointer(np.uintp, flags="C_CONTIGUOUS")
sz = ctypes.c_size_t


class AttnWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "q_norm", "k_norm",
                                               "o_w", "o_b")]


def _cpu_signature() -> str:
    """Model name + ISA flags of this host: the library is built with
    -march=native, so a copy built on another CPU is rebuilt before use."""
    try:
        text = pathlib.Path("/proc/cpuinfo").read_text()
    except OSError:
        return "unknown"
    model = next((l for l in text.splitlines() if l.startswith("model name")), "")
    flags = next((l for l in text.splitlines() if l.startswith("flags")), "")
    return f"{model}|{flags}"


def build() -> pathlib.Path:
    """Builds the oracle library with make if it is missing, stale, or was
    built on a different CPU."""
    src = [HERE / "ncm_oracle.cpp", HERE / "ncm_oracle.h", HERE / "Makefile"]
    stamp = HERE / "build" / "cpu.stamp"
    sig = _cpu_signature()
    stale = not LIB.exists() or LIB.stat().st_mtime < max(s.stat().st_mtime for s in src)
    foreign = not stamp.exists() or stamp.read_text() != sig
    if stale or foreign:
        subprocess.run(["make", "-s", "-B", "-C", os.fspath(HERE)], check=True)
        stamp.write_text(sig)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    build()
    L = ctypes.CDLL(os.fspath(LIB))
    sig = {
        "orc_bf16_from_f32": ([ctypes.c_float], ctypes.c_uint16),
        "orc_bf16_to_f32": ([ctypes.c_uint16], ctypes.c_float),
        "orc_bf16_from_f32_n": ([f32p, u16p, sz], None),
        "orc_round_bf16_n": ([f32p, f32p, sz], None),
        "orc_matmul": ([f32p, f32p, f32p, sz, sz, sz], None),
        "orc_matmul_reference": ([f32p, f32p, f32p, sz, sz, sz], None),
        "orc_matmul_bf16": ([f32p, f32p, ctypes.c_void_p, f32p, sz, sz, sz], None),
        "orc_matmul_bf16_mt": ([f32p, f32p, ctypes.c_void_p, f32p, sz, sz, sz, ctypes.c_int], None),
        "orc_sum_squares_pinned": ([f32p, sz], ctypes.c_float),
        "orc_rms_norm": ([f32p, f32p, f32p, sz, ctypes.c_float], None),
        "orc_rms_norm_bf16": ([f32p, f32p, f32p, sz, ctypes.c_float], None),
        "orc_silu": ([f32p, f32p, sz], None),
        "orc_silu_bf16": ([f32p, f32p, sz], None),
        "orc_softmax": ([f32p, f32p, sz], None),
        "orc_rms_norm_rows": ([f32p, f32p, ctypes.c_void_p, f32p, sz, sz, ctypes.c_float], None),
        "orc_rope_default": ([sz, ctypes.c_float, sz, f32p, f32p, f32p], None),
        "orc_rope_tables": ([f32p, sz, sz, f32p, f32p], None),
        "orc_rope_llama3": ([sz, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, sz, f32p], None),
        "orc_causal_mask": ([szp, sz, szp, sz, ctypes.c_long, u8p], None),
        "orc_block_diagonal_mask": ([sz, szp, sz, ctypes.c_void_p, sz, u8p, sz], ctypes.c_int),
        "orc_block_causal_mask": ([sz, szp, sz, ctypes.c_void_p, sz, u8p, sz], ctypes.c_int),
        "orc_fill_level_positions": ([sz, szp, sz, szp, sz], ctypes.c_int),
        "orc_apply_post_upsample_conv": ([f32p, f32p, f32p, sz, sz], ctypes.c_int),
        "orc_attention": ([f32p, ctypes.POINTER(AttnWeights), sz, sz, sz, sz, sz, ctypes.c_float, f32p, f32p, u8p,
                           f32p, ctypes.c_int, ctypes.c_void_p], ctypes.c_int),
        "orc_attention_core_rows": ([f32p, f32p, f32p, u8p, sz, sz, sz, sz, sz, f32p, ctypes.c_int, ctypes.c_int],
                                    ctypes.c_int),
        "orc_rotate_rows": ([f32p, sz, sz, sz, f32p, f32p, ctypes.c_int], None),
        "orc_code_sqnorm": ([u16p, f32p, sz, sz], None),
        "orc_rvq_level": ([f32p, u16p, f32p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, sz, sz, sz,
                           ctypes.c_int], None),
        "orc_rvq_decode": ([i32p, u16p, sz, f32p, sz, sz, sz], None),
        "orc_pool_avg": ([f32p, f32p, sz, sz, sz, sz], None),
        "orc_scale_update": ([i32p, u16p, sz, f32p, f32p, sz, sz, sz, sz, sz], None),
        "orc_tied_head": ([f32p, u16p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p,
                           ctypes.c_void_p, ctypes.c_void_p, sz, sz, sz], None),
        "orc_group_norm": ([f32p, f32p, sz, sz, sz, sz, ctypes.c_float], None),
        "orc_conv_down4": ([f32p, f32p, ctypes.c_void_p, f32p, sz, sz, sz], None),
        "orc_conv_up4": ([f32p, f32p, ctypes.c_void_p, f32p, sz, sz, sz], None),
        "orc_ema": ([f32p, i32p, sz, sz, sz, f32p, f32p, f32p, ctypes.c_float, ctypes.c_float, ctypes.c_void_p,
                     ctypes.c_void_p], None),
        "orc_upsample": ([f32p, f32p, sz, sz, sz, sz, ctypes.c_int], None),
        "orc_conv1d_k3": ([f32p, ctypes.c_void_p, f32p, ctypes.c_void_p, f32p, sz, sz, ctypes.c_void_p, sz,
                           ctypes.c_float, ctypes.c_float], None),
        "orc_scale_update_ex": ([i32p, u16p, sz, ctypes.c_void_p, f32p, sz, sz, sz, sz, sz, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _vp(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------ bf16
def bf16_bits(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_bf16_from_f32_n(x.ravel(), out.ravel(), x.size)
    return out


def bf16_widen(b: np.ndarray) -> np.ndarray:
    return (_c(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_widen(bf16_bits(x))


# --------------------------------------------------------------- linears
def matmul_bf16(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None, threads: int = 1) -> np.ndarray:
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    T, K = x.shape
    N = w.shape[0]
    out = np.empty((T, N), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    if threads > 1:
        lib().orc_matmul_bf16_mt(x, w, _vp(b), out, T, K, N, threads)
    else:
        lib().orc_matmul_bf16(x, w, _vp(b), out, T, K, N)
    return out


def matmul(x: np.ndarray, w: np.ndarray, reference: bool = False) -> np.ndarray:
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    T, K = x.shape
    N = w.shape[0]
    out = np.empty((T, N), np.float32)
    (lib().orc_matmul_reference if reference else lib().orc_matmul)(x, w, out, T, K, N)
    return out


# ------------------------------------------------------------ elementwise
def sum_squares_pinned(x: np.ndarray) -> np.float32:
    x = _c(x, np.float32)
    return np.float32(lib().orc_sum_squares_pinned(x, x.size))


def _unary(name, x):
    x = _c(x, np.float32)
    out = np.empty_like(x)
    getattr(lib(), name)(x.ravel(), out.ravel(), x.size)
    return out


def silu(x):
    return _unary("orc_silu", x)


def silu_bf16(x):
    return _unary("orc_silu_bf16", x)


def softmax(x):
    return _unary("orc_softmax", x)


def rms_norm(x, w, eps, bf16_mode=False):
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    out = np.empty_like(x)
    (lib().orc_rms_norm_bf16 if bf16_mode else lib().orc_rms_norm)(x, w, out, x.size, eps)
    return out


def rms_norm_rows(x, w, eps, bias=None):
    x = _c(x, np.float32)
    rows, width = x.shape
    out = np.empty_like(x)
    b = None if bias is None else _c(bias, np.float32)
    lib().orc_rms_norm_rows(x, _c(w, np.float32), _vp(b), out, rows, width, eps)
    return out


# ------------------------------------------------------------ rope / masks
def rope_default(head_dim, theta, positions):
    inv = np.empty(head_dim // 2, np.float32)
    c = np.empty((positions, head_dim), np.float32)
    s = np.empty((positions, head_dim), np.float32)
    lib().orc_rope_default(head_dim, theta, positions, inv, c, s)
    return inv, c, s


def rope_tables(inv_freq, positions):
    inv = _c(inv_freq, np.float32)
    hd = inv.size * 2
    c = np.empty((positions, hd), np.float32)
    s = np.empty((positions, hd), np.float32)
    lib().orc_rope_tables(inv, inv.size, positions, c, s)
    return c, s


def rope_llama3(head_dim, theta, factor, low, high, orig):
    inv = np.empty(head_dim // 2, np.float32)
    lib().orc_rope_llama3(head_dim, theta, factor, low, high, orig, inv)
    return inv


def causal_mask(qpos, kpos, window=0):
    q = _c(qpos, np.uintp)
    k = _c(kpos, np.uintp)
    out = np.empty((q.size, k.size), np.uint8)
    lib().orc_causal_mask(q, q.size, k, k.size, int(window or 0), out)
    return out.astype(bool)


def _level_mask(fn, prefix, levels, pad_mask):
    lv = _c(levels, np.uintp)
    S = prefix + int(lv.sum())
    out = np.empty((S, S), np.uint8)
    pm = None if pad_mask is None or len(pad_mask) == 0 else _c(pad_mask, np.uint8)
    rc = fn(prefix, lv, lv.size, _vp(pm), 0 if pm is None else pm.size, out, out.size)
    if rc != 0:
        raise ValueError(f"mask construction failed ({rc})")
    return out.astype(bool)


def block_diagonal_mask(prefix, levels, pad_mask=None):
    return _level_mask(lib().orc_block_diagonal_mask, prefix, levels, pad_mask)


def block_causal_mask(prefix, levels, pad_mask=None):
    return _level_mask(lib().orc_block_causal_mask, prefix, levels, pad_mask)


def fill_level_positions(prefix, levels):
    lv = _c(levels, np.uintp)
    out = np.empty(prefix + int(lv.sum()), np.uintp)
    if lib().orc_fill_level_positions(prefix, lv, lv.size, out, out.size) != 0:
        raise ValueError("bad position buffer")
    return out


def apply_post_upsample_conv(x, w, b):
    x = _c(x, np.float32).copy()
    rows, width = x.shape
    lib().orc_apply_post_upsample_conv(x, _c(w, np.float32), _c(b, np.float32), rows, width)
    return x


def attention(x, weights: dict, heads, kv_heads, head_dim, eps, cos_t, sin_t, mask, bf16_mode=False):
    x = _c(x, np.float32)
    T, hidden = x.shape
    keep = {}
    w = AttnWeights()
    for name in ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "q_norm", "k_norm", "o_w", "o_b"):
        a = weights.get(name)
        if a is not None:
            keep[name] = _c(a, np.float32)
            setattr(w, name, keep[name].ctypes.data)
    out = np.empty((T, hidden), np.float32)
    rc = lib().orc_attention(x, ctypes.byref(w), T, hidden, heads, kv_heads, head_dim, eps, _c(cos_t, np.float32),
                             _c(sin_t, np.float32), _c(mask, np.uint8), out, int(bf16_mode), None)
    if rc != 0:
        raise ValueError("attention: bad arguments")
    return out


def attention_rows(x, weights: dict, heads, kv_heads, head_dim, cos_t, sin_t, mask, rows, bf16_mode=True,
                   threads=1):
    """attention_impl (packages/kernels/root.zig:450-581) for the query rows
    `rows` only: K and V are projected for every row of x, Q for the chosen
    rows; each returned row [len(rows), hidden] has the bits orc_attention
    gives that row (no biases, no QK-norm). cos_t/sin_t [T, head_dim], mask
    [T, T]."""
    x = _c(x, np.float32)
    rows = np.asarray(rows, np.int64)
    T, hidden = x.shape
    # project (root.zig:583-609): matmul_bf16 in bf16 mode, else the f32 32-tile matmul
    proj = (lambda a, w: matmul_bf16(a, w, threads=threads)) if bf16_mode else matmul  # noqa: E731
    q = proj(x[rows], weights["q_w"])
    k = proj(x, weights["k_w"])
    v = proj(x, weights["v_w"])
    cos_t, sin_t = _c(cos_t, np.float32), _c(sin_t, np.float32)
    lib().orc_rotate_rows(q, rows.size, heads, head_dim, _c(cos_t[rows], np.float32), _c(sin_t[rows], np.float32),
                          int(bf16_mode))
    lib().orc_rotate_rows(k, T, kv_heads, head_dim, cos_t, sin_t, int(bf16_mode))
    ctx = np.empty((rows.size, heads * head_dim), np.float32)
    rc = lib().orc_attention_core_rows(q, k, v, _c(np.asarray(mask)[rows], np.uint8), rows.size, T, heads, kv_heads,
                                       head_dim, ctx, int(bf16_mode), threads)
    if rc != 0:
        raise ValueError("attention_rows: bad arguments")
    return proj(ctx, weights["o_w"])


# ------------------------------------------------------------------- RVQ
def code_sqnorm(cb_bits: np.ndarray) -> np.ndarray:
    cb = _c(cb_bits, np.uint16)
    D = cb.shape[-1]
    K = cb.size // D
    out = np.empty(cb.shape[:-1], np.float32)
    lib().orc_code_sqnorm(cb.ravel(), out.ravel(), K, D)
    return out


def rvq_level(resid: np.ndarray, cb_bits: np.ndarray, sqnorm: np.ndarray, codes_in: np.ndarray | None = None,
              threads: int = 0):
    """One level; updates `resid` (f32 [N, D]) in place. Returns (best codes, relative top-2 gap)."""
    assert resid.dtype == np.float32 and resid.flags.c_contiguous
    N, D = resid.shape
    cb = _c(cb_bits, np.uint16)
    K = cb.shape[0]
    best = np.empty(N, np.int32)
    gap = np.empty(N, np.float32)
    ci = None if codes_in is None else _c(codes_in, np.int32)
    th = threads or (os.cpu_count() or 1)
    lib().orc_rvq_level(resid, cb, _c(sqnorm, np.float32), _vp(ci), _vp(best), _vp(gap), N, D, K, th)
    return best, gap


def rvq_decode(codes: np.ndarray, cbs_bits: np.ndarray) -> np.ndarray:
    codes = _c(codes, np.int32)
    cbs = _c(cbs_bits, np.uint16)
    L, N = codes.shape
    _, K, D = cbs.shape
    out = np.empty((N, D), np.float32)
    lib().orc_rvq_decode(codes, cbs, L, out, N, D, K)
    return out


def pool_avg(x: np.ndarray, f: int) -> np.ndarray:
    x = _c(x, np.float32)
    B, T, D = x.shape
    y = np.empty((B, T // f, D), np.float32)
    lib().orc_pool_avg(x, y, B, T, D, f)
    return y


def scale_update(codes: np.ndarray, cbs_bits: np.ndarray, resid: np.ndarray, recon: np.ndarray, B, T, f):
    L, P = codes.shape
    _, K, D = cbs_bits.shape
    assert resid.dtype == np.float32 and recon.dtype == np.float32
    lib().orc_scale_update(_c(codes, np.int32), _c(cbs_bits, np.uint16), L, resid, recon, B, T, D, K, f)


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def tied_head(z, cb_bits, log_inv_T=0.0, bias=None, esq=None, want_logits=True):
    """_TiedCodebookHead: returns (logits [T, K] or None, argmax codes [T], top-2 logit gap [T])."""
    z = _c(z, np.float32)
    T, d = z.shape
    cb_bits = _c(cb_bits, np.uint16)
    K = cb_bits.shape[0]
    bias = None if bias is None else _c(bias, np.float32)
    esq = None if esq is None else _c(esq, np.float32)
    logits = np.empty((T, K), np.float32) if want_logits else None
    codes = np.empty(T, np.int32)
    gap = np.empty(T, np.float32)
    lib().orc_tied_head(z, cb_bits, _ptr(esq), _ptr(bias), log_inv_T, _ptr(logits), _ptr(codes), _ptr(gap), T, d, K)
    return logits, codes, gap


def group_norm(x, groups, eps=1e-5):
    x = _c(x, np.float32)
    B, T, C = x.shape
    y = np.empty_like(x)
    lib().orc_group_norm(x, y, B, T, C, groups, eps)
    return y


def conv_down4(x, w, b=None):
    """Conv1d(C, C, 4, stride 4) over axis 1 of x [B, L, C]; w [C, C, 4]."""
    x = _c(x, np.float32)
    B, L, C = x.shape
    y = np.empty((B, L // 4, C), np.float32)
    lib().orc_conv_down4(x, _c(w, np.float32), _ptr(None if b is None else _c(b, np.float32)), y, B, L, C)
    return y


def conv_up4(x, w, b=None):
    """ConvTranspose1d(C, C, 4, stride 4) over axis 1 of x [B, L, C]; w [C_in, C_out, 4]."""
    x = _c(x, np.float32)
    B, L, C = x.shape
    y = np.empty((B, 4 * L, C), np.float32)
    lib().orc_conv_up4(x, _c(w, np.float32), _ptr(None if b is None else _c(b, np.float32)), y, B, L, C)
    return y


def ema(u, codes, ema_count, ema_sum, decay, eps):
    """One EMA step; returns (ema_count, ema_sum, codebook, counts, sums) as new arrays."""
    u = _c(u, np.float32)
    N, D = u.shape
    K = ema_count.shape[0]
    cnt = _c(ema_count, np.float32).copy()
    sm = _c(ema_sum, np.float32).copy()
    cb = np.empty((K, D), np.float32)
    counts = np.empty(K, np.float32)
    sums = np.empty((K, D), np.float32)
    lib().orc_ema(u, _c(codes, np.int32), N, D, K, cnt, sm, cb, decay, eps, _ptr(counts), _ptr(sums))
    return cnt, sm, cb, counts, sums


def upsample(q: np.ndarray, T: int, mode: str = "linear") -> np.ndarray:
    """F.interpolate(size=T) along axis 1 of q [B, Tq, D] (nearest / linear, align_corners=False)."""
    q = _c(q, np.float32)
    B, Tq, D = q.shape
    out = np.empty((B, T, D), np.float32)
    lib().orc_upsample(q, out, B, Tq, T, D, {"nearest": 0, "linear": 1}[mode])
    return out


def conv1d_k3(x_op, w, b, segments=None, alpha=1.0, beta=1.0, x_blend=None):
    """out = alpha * x_blend + beta * (b + conv(x_op; w)) per row segment (f64 accumulation)."""
    x_op = _c(x_op, np.float32)
    rows, width = x_op.shape
    x_blend = x_op if x_blend is None else _c(x_blend, np.float32)
    w = _c(w, np.float32)
    b = None if b is None else _c(b, np.float32)
    segs = None if segments is None else np.ascontiguousarray(segments, dtype=np.uintp)
    out = np.empty((rows, width), np.float32)
    lib().orc_conv1d_k3(x_op, _ptr(x_blend), w, _ptr(b), out, rows, width, _ptr(segs),
                        0 if segs is None else len(segs), alpha, beta)
    return out


def scale_update_ex(codes, cbs_bits, resid, acc, B, T, f, mode="nearest", phi_w=None, phi_b=None, ratio=0.5):
    """General multiscale step (upsampling mode, optional Phi); updates resid (may be None) and acc in place."""
    L, P = codes.shape
    _, K, D = cbs_bits.shape
    assert acc.dtype == np.float32 and (resid is None or resid.dtype == np.float32)
    phi_w = None if phi_w is None else _c(phi_w, np.float32)
    phi_b = None if phi_b is None else _c(phi_b, np.float32)
    lib().orc_scale_update_ex(_c(codes, np.int32), _c(cbs_bits, np.uint16), L, _ptr(resid), acc, B, T, D, K, f,
                              {"nearest": 0, "linear": 1}[mode], _ptr(phi_w), _ptr(phi_b), ratio)


def rvq_encode(x_bits: np.ndarray, cbs_bits: np.ndarray, codes_in: np.ndarray | None = None, threads: int = 0):
    """L levels over bf16 x. With codes_in [L, N] the residual follows those codes
    (teacher forcing). Returns (oracle best codes [L, N], gaps [L, N], residual, recon f32)."""
    x = bf16_widen(x_bits).astype(np.float32).copy()
    L, K, D = cbs_bits.shape
    N = x.shape[0]
    best = np.empty((L, N), np.int32)
    gaps = np.empty((L, N), np.float32)
    sq = code_sqnorm(cbs_bits)
    for l in range(L):
        ci = None if codes_in is None else codes_in[l]
        best[l], gaps[l] = rvq_level(x, cbs_bits[l], sq[l], ci, threads)
    used = best if codes_in is None else codes_in
    recon = rvq_decode(used, cbs_bits)
    return best, gaps, x, recon
