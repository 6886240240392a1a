"""ctypes binding of libncm_cuda.so (the C ABI declared in include/ncm_cuda.h).

The library is loaded from this package directory only. There is no fallback:
if the shared object is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "libncm_cuda.so"

NCM_OK = 0
NCM_EINVAL = -1
NCM_ECUDA = -2
NCM_ENOMEM = -3
NCM_ETIMEOUT = -4
NCM_ERANGE = -5
NCM_ENOTSUP = -6

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p


class TokenizerConfig(ctypes.Structure):
    """Mirror of ncm_tokenizer_config_t."""

    _fields_ = [
        ("batch", c_i64),
        ("seq_len", c_i64),
        ("model_width", c_i64),
        ("vq_width", c_i64),
        ("codebook_size", c_i64),
        ("num_scales", c_i32),
        ("levels_per_scale", c_i32),
        ("pool_factors", c_i32 * 16),
        ("upsample_mode", c_i32),
        ("phi_ratio", ctypes.c_float),
    ]


class Mask(ctypes.Structure):
    """Mirror of ncm_mask_t."""

    _fields_ = [
        ("mode", c_i32),
        ("prefix_length", c_i32),
        ("prefix_pad_mask", ctypes.c_uint64),
        ("num_levels", c_i32),
        ("level_lengths", c_i32 * 32),
        ("sliding_window", c_i32),
    ]


class IpcHandle(ctypes.Structure):
    """Mirror of ncm_ipc_handle_t."""

    _fields_ = [("handle", ctypes.c_uint8 * 64), ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


class DecoderConfig(ctypes.Structure):
    """Mirror of ncm_decoder_config_t."""

    _fields_ = [
        ("hidden_size", c_i64),
        ("vq_width", c_i64),
        ("num_attention_heads", c_i64),
        ("num_key_value_heads", c_i64),
        ("head_dim", c_i64),
        ("intermediate_size", c_i64),
        ("rms_norm_epsilon", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("use_level_encoding", c_i32),
        ("mask", Mask),
        ("rope_type", c_i32),
        ("rope_factor", ctypes.c_float),
        ("rope_low_freq_factor", ctypes.c_float),
        ("rope_high_freq_factor", ctypes.c_float),
        ("rope_original_max_position_embeddings", c_i64),
    ]


class DecoderLayerWeights(ctypes.Structure):
    """Mirror of ncm_decoder_layer_weights_t (device pointers)."""

    _fields_ = [(n, c_vp) for n in ("ln_1", "qkv", "qkv_bias", "o", "o_bias", "ln_2", "gate_up", "down", "q_norm",
                                    "k_norm")]


class DecoderWeights(ctypes.Structure):
    """Mirror of ncm_decoder_weights_t."""

    _fields_ = [
        ("input_projection", c_vp),
        ("input_projection_bias", c_vp),
        ("level_embedding", c_vp),
        ("final_norm", c_vp),
        ("final_norm_bias", c_vp),
        ("num_layers", c_i32),
        ("layers", ctypes.POINTER(DecoderLayerWeights)),
        ("post_conv_weight", c_vp),
        ("post_conv_bias", c_vp),
    ]


# name -> argtypes (all functions return int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "ncm_ctx_create": [ctypes.c_int, ctypes.POINTER(c_vp)],
    "ncm_ctx_destroy": [c_vp],
    "ncm_sync": [c_vp, c_vp],
    "ncm_status_string": [ctypes.c_int],
    "ncm_last_error": [],
    "ncm_version": [],
    "ncm_f32_to_bf16": [c_vp, c_vp, c_vp, c_i64, c_vp],
    "ncm_bf16_to_f32": [c_vp, c_vp, c_vp, c_i64, c_vp],
    "ncm_linear_bf16": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_linear_bf16_host_f32": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64],
    "ncm_matmul_host_f32": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64],
    "ncm_code_sqnorm": [c_vp, c_vp, c_vp, c_i64, c_i64, c_vp],
    "ncm_rvq_level": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_rvq_encode": [c_vp, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_rvq_encode_host": [c_vp, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_pool_avg": [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_vp],
    "ncm_rvq_decode": [c_vp, c_vp, c_vp, c_i32, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_rms_norm_bf16": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, ctypes.c_float, c_vp],
    "ncm_embedding_gather": [c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp],
    "ncm_rope_tables_host": [c_i32, ctypes.c_float, c_vp, c_i64, c_vp, c_vp],
    "ncm_rope_tables_llama3_host": [c_i32, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, c_i64,
                                    c_vp, c_i64, c_vp, c_vp],
    "ncm_attention_bf16": [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, ctypes.POINTER(Mask), c_vp],
    "ncm_attention_qk_norm_bf16": [c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, ctypes.c_float, c_vp, c_i64, c_i32, c_i32,
                                   ctypes.POINTER(Mask), c_vp],
    "ncm_ncm_forward": [c_vp, ctypes.POINTER(DecoderConfig), ctypes.POINTER(DecoderWeights), c_vp, c_vp, c_vp],
    "ncm_rvq_level_noalloc": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_rvq_level_noalloc_status": [c_vp, ctypes.POINTER(c_i32)],
    "ncm_profile_enable": [c_vp, ctypes.c_int],
    "ncm_profile_read": [c_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_i64)],
    "ncm_tokenizer_forward": [c_vp, ctypes.POINTER(TokenizerConfig), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                              c_vp, c_vp, c_vp, c_vp],
    "ncm_tokenizer_forward_ex": [c_vp, ctypes.POINTER(TokenizerConfig), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                 c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "ncm_multiscale_decode": [c_vp, ctypes.POINTER(TokenizerConfig), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "ncm_rvq_level_top2": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_tied_head_logits": [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_float, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_tied_head_argmax": [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_float, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_comm_unique_id": [c_vp],
    "ncm_ctx_comm_init": [c_vp, c_vp, c_i32, c_i32],
    "ncm_ipc_export": [c_vp, ctypes.c_uint64, ctypes.POINTER(IpcHandle)],
    "ncm_ipc_open": [ctypes.POINTER(IpcHandle), ctypes.POINTER(c_vp)],
    "ncm_ipc_close": [c_vp],
    "ncm_copy_async": [c_vp, c_vp, ctypes.c_uint64, c_vp],
    "ncm_copy2d_async": [c_vp, ctypes.c_uint64, c_vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, c_vp],
    "ncm_rvq_encode_sharded": [c_vp, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_load_tensor_bf16": [c_vp, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_uint64, c_i32, c_vp, c_vp],
    "ncm_qkv_projection_rope": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i32, c_i32, c_vp],
    "ncm_group_norm": [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, ctypes.c_float, c_vp],
    "ncm_conv_down4": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_conv_up4": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_ema_code_stats": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp],
    "ncm_ema_update": [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, ctypes.c_float, ctypes.c_float, c_vp],
    "ncm_upsample": [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp],
    "ncm_conv1d_k3": [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i32, c_vp, ctypes.c_float, ctypes.c_float,
                      c_vp],
    "ncm_post_upsample_conv_host_f32": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64],
}
_RESTYPES = {"ncm_status_string": ctypes.c_char_p, "ncm_last_error": ctypes.c_char_p}

_lib = None


class NcmError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"ncm status {status}: {message}")
        self.status = status


def load() -> ctypes.CDLL:
    """Loads libncm_cuda.so from the package directory (raises if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m ncmorph_b200.build` (there is no CPU fallback)")
    lib = ctypes.CDLL(os.fspath(LIB_PATH), mode=ctypes.RTLD_LOCAL)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != NCM_OK:
        msg = load().ncm_last_error()
        raise NcmError(status, msg.decode(errors="replace") if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
