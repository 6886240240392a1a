"""ncmorph_b200: B200-native (sm_100a) kernels for ncmorph's quantisation hot
path — the multiscale residual-VQ tokenizer forward and the bf16 linear
layers — behind a C ABI (include/ncm_cuda.h, libncm_cuda.so).

libncm_cuda.so is loaded on first use (``ncmorph_b200._lib.load()``); if it
is missing every entry point raises ImportError. There is no CPU fallback.
"""
from . import device, kernels, ncm_model, vq  # noqa: F401

__all__ = ["device", "kernels", "ncm_model", "vq"]
