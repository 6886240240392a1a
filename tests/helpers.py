"""Helpers shared by the GPU parity tests: seeded synthetic inputs and the
parity rules.

Parity rules (the bars the kernels are held to):
  * integer codes: bit-exact, except rows whose oracle top-2 distance gap is
    below NEAR_TIE relative to the best full squared distance; those rows are
    counted as near-ties and their flips reported, never hidden;
  * bf16 outputs of GEMMs: |gpu - oracle| <= BF16_REL * |oracle| + ACC_ABS *
    sum_k |x_k w_k| (one bf16 rounding flip plus f32 accumulation-order noise);
  * everything whose inputs are identical on both sides (residual updates,
    decode, pooling, code norms) is compared bit for bit.
"""
from __future__ import annotations

import numpy as np
import torch

NEAR_TIE = 1e-3
BF16_REL = 2e-2
ACC_ABS = 1e-5


def gen_bf16(rng: np.random.Generator, shape, scale=1.0) -> np.ndarray:
    """N(0, scale^2) in f32, rounded to bf16 bits with the reference rule."""
    from oracle import pyoracle as orc
    return orc.bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def to_dev_bf16(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def from_dev_bf16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def check_codes(gpu: np.ndarray, oracle_best: np.ndarray, gap: np.ndarray, what: str) -> dict:
    """Codes must agree wherever the oracle's top-2 gap is >= NEAR_TIE."""
    far = gap >= NEAR_TIE
    mism = gpu != oracle_best
    bad = np.nonzero(mism & far)[0]
    assert bad.size == 0, (f"{what}: {bad.size} code mismatches outside near-ties, first row {bad[0]} "
                           f"gpu={gpu[bad[0]]} oracle={oracle_best[bad[0]]} gap={gap[bad[0]]}")
    return {"rows": int(gpu.size), "near_ties": int((~far).sum()), "flips": int(mism.sum())}


def check_free_running(gpu: np.ndarray, free_best: np.ndarray, tf_gap: np.ndarray, what: str) -> dict:
    """Free-running comparison over L levels ([L, n] codes): the oracle encodes
    the rows on its own (free_best), so a near-tie flip at one level changes
    the residual and may change every later level. Each row that diverges
    must do so first at a level whose gap is below NEAR_TIE; until that level
    both histories are identical, so the teacher-forced oracle's gap there
    (tf_gap) is the free-running oracle's too."""
    L, n = gpu.shape
    differ = gpu != free_best
    diverged = differ.any(axis=0)
    first = np.where(diverged, differ.argmax(axis=0), -1)
    rows = np.nonzero(diverged)[0]
    gaps_at_first = tf_gap[first[rows], rows]
    bad = rows[gaps_at_first >= NEAR_TIE]
    assert bad.size == 0, (f"{what}: row {bad[0]} first diverges at level {first[bad[0]]} where the gap is "
                           f"{tf_gap[first[bad[0]], bad[0]]} (not a near-tie)")
    return {"rows": int(n), "diverged_rows": int(rows.size), "codes_differing": int(differ.sum()),
            "first_divergence_levels": np.bincount(first[rows], minlength=L).tolist()}


def check_gemm(y: np.ndarray, ref: np.ndarray, absprod: np.ndarray, what: str) -> float:
    tol = BF16_REL * np.abs(ref) + ACC_ABS * absprod
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    bad = np.argwhere(err > tol)
    assert bad.size == 0, f"{what}: {len(bad)} elements outside tolerance, first {bad[0]} y={y[tuple(bad[0])]} ref={ref[tuple(bad[0])]}"
    return float((err / np.maximum(np.abs(ref), 1e-30)).max())
