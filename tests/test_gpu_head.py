"""GPU parity of the codebook-tied output head (_TiedCodebookHead,
PROJECT.md:222) against the CPU oracle, through the C ABI.

Logits: the dot products accumulate in a different order on the tensor cores
(f32) than in the oracle (exact f64, rounded once), so the bar is the GEMM
bar carried through the head's affine map:
|gpu - oracle| <= 1e-5 * e / d_scale * (2 sum|z e| + E_sq) + 1e-6 |oracle|.
Argmax codes: bit-exact outside near-ties (oracle top-2 logit gap below
1e-4 * max(1, |best|)); the upstream module is not vendored, so the head's
parity is against the oracle's restatement only (unpinned).
"""
import numpy as np
import pytest
import torch

from helpers import from_dev_bf16, gen_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def _case(orc, rng, T, d, K, with_bias):
    z = gen_bf16(rng, (T, d))
    cb = gen_bf16(rng, (K, d))
    bias = (rng.standard_normal(K) * 0.05).astype(np.float32) if with_bias else None
    return z, cb, bias


@pytest.mark.parametrize("T,d,K,with_bias,lit", [
    (1024, 384, 8192, True, 0.0),     # OWT head shape: d = 384, K = 8192, one level of 1024 positions
    (100, 64, 700, False, 0.7),       # one row block (code-split argmax), K not a multiple of 256
    (148 * 128, 136, 512, True, -0.3),  # row blocks fill the GPU (no split), d not a multiple of 64
    (1, 8, 5, True, 0.0),             # smallest legal head
])
def test_tied_head_logits_and_argmax(orc, cuda_dev, T, d, K, with_bias, lit):
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(T + d + K)
    z, cb, bias = _case(orc, rng, T, d, K, with_bias)
    zd, cbd = to_dev_bf16(z, cuda_dev), to_dev_bf16(cb, cuda_dev)
    bd = None if bias is None else torch.from_numpy(bias).to(cuda_dev)
    logits = ncm_model.tied_head_logits(zd, cbd, lit, bd).cpu().numpy()
    codes = ncm_model.tied_head_argmax(zd, cbd, lit, bd).cpu().numpy()
    zf = orc.bf16_widen(z).astype(np.float32)
    sample = np.arange(T) if T <= 2048 else np.sort(rng.choice(T, 2048, replace=False))
    ref, best, gap = orc.tied_head(zf[sample], cb, lit, bias)
    ef = orc.bf16_widen(cb).astype(np.float64)
    esq = (ef ** 2).sum(1)
    scale = np.exp(lit) / esq.mean()
    bound = 1e-5 * scale * (2 * np.abs(zf[sample]).astype(np.float64) @ np.abs(ef).T + esq) + 1e-6 * np.abs(ref)
    err = np.abs(logits[sample].astype(np.float64) - ref)
    assert np.all(err <= bound), err.max()
    far = gap >= 1e-4 * np.maximum(1.0, np.abs(ref.max(axis=1)))
    assert np.array_equal(codes[sample][far], best[far])
    print(f"T={T} K={K}: near-ties {int((~far).sum())} of {len(sample)}, flips {int((codes[sample] != best).sum())}")


def test_tied_head_argmax_equals_rvq_argmin_without_bias(cuda_dev):
    """With no bias the head's argmax is the nearest codeword: the RVQ code."""
    from ncmorph_b200 import ncm_model, vq
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    z = torch.randn((4096, 256), generator=g, device=cuda_dev).to(torch.bfloat16)
    cb = torch.randn((4096, 256), generator=g, device=cuda_dev).to(torch.bfloat16)
    head = ncm_model.tied_head_argmax(z, cb, 0.0)
    r = z.float()
    rvq = vq.rvq_level(r, cb)
    assert (head == rvq).float().mean().item() > 0.999


def test_tied_head_rejects_bad_width(cuda_dev):
    from ncmorph_b200 import _lib, ncm_model
    z = torch.zeros((4, 12), dtype=torch.bfloat16, device=cuda_dev)
    cb = torch.zeros((8, 12), dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(_lib.NcmError) as ei:
        ncm_model.tied_head_logits(z, cb)
    assert ei.value.status == _lib.NCM_EINVAL
