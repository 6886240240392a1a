"""GPU parity of the time upsampling (R5 modes) and of the kernel-3
convolution (the quantiser's Phi and ncm_model.apply_post_upsample_conv)
against the CPU oracle, through the C ABI.

Upsampling has no arithmetic freedom: it is compared bit for bit (the oracle
itself is pinned bit-exact to torch's F.interpolate). The convolution sums on
the tensor cores with bf16 operands; its bar is the GEMM bar on the same
bf16 operand values, |gpu - oracle| <= 1e-5 * sum |w x| + 1e-6 |oracle|.
"""
import numpy as np
import pytest
import torch

from helpers import to_dev_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,Tq,D,T", [(8, 128, 1024, 2048), (2, 37, 24, 100), (3, 1, 8, 16), (1, 64, 64, 64),
                                      (4, 256, 128, 512)])
@pytest.mark.parametrize("mode", ["linear", "nearest"])
def test_upsample_bit_exact(orc, cuda_dev, B, Tq, D, T, mode):
    from ncmorph_b200 import vq
    q = np.random.default_rng(B * Tq + T).standard_normal((B, Tq, D)).astype(np.float32)
    got = vq.upsample(torch.from_numpy(q).to(cuda_dev), T, mode).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), orc.upsample(q, T, mode).view(np.uint32))


def _conv_case(orc, rng, rows, width, segments, alpha, beta, wscale=0.05):
    x = rng.standard_normal((rows, width)).astype(np.float32)
    w_bits = orc.bf16_bits((rng.standard_normal((width, width, 3)) * wscale).astype(np.float32))
    b = (rng.standard_normal(width) * 0.1).astype(np.float32)
    w = orc.bf16_widen(w_bits)
    ref = orc.conv1d_k3(orc.round_bf16(x), w, b, segments=segments, alpha=alpha, beta=beta, x_blend=x)
    # sum |w||x| over the taps that fall inside each row's segment (upper bound: all taps)
    ax = np.abs(orc.round_bf16(x))
    sw = np.abs(w).sum(axis=2)
    absprod = ax @ sw.T
    absprod[1:] += ax[:-1] @ sw.T
    absprod[:-1] += ax[1:] @ sw.T
    return x, w_bits, b, ref, np.abs(beta) * (absprod + np.abs(b))


@pytest.mark.parametrize("rows,width,segments,alpha,beta", [
    (300, 64, None, 1.0, 1.0),                  # apply_post_upsample_conv form, 3 row tiles
    (1000, 136, [100, 300, 600], 0.5, 0.5),     # unequal segments, width not a multiple of 64
    (4096, 1024, [2048, 2048], 0.5, 0.5),       # Phi at the tokenizer's width, two batch items
    (5, 24, None, 1.0, 1.0),                    # fewer rows than one tile
    (700, 64, [7] * 100, 0.25, 0.75),           # 100 equal segments (closed-form row map)
])
def test_conv1d_k3_matches_oracle(orc, cuda_dev, rows, width, segments, alpha, beta):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(rows + width)
    x, w_bits, b, ref, bound = _conv_case(orc, rng, rows, width, segments, alpha, beta)
    xd = torch.from_numpy(x).to(cuda_dev)
    got = vq.conv1d_k3(xd, to_dev_bf16(w_bits, cuda_dev), torch.from_numpy(b).to(cuda_dev), segments=segments,
                       alpha=alpha, beta=beta).cpu().numpy()
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= 1e-5 * bound + 1e-6 * np.abs(ref)), err.max()
    # in place (out is x) gives the same values
    vq.conv1d_k3(xd, to_dev_bf16(w_bits, cuda_dev), torch.from_numpy(b).to(cuda_dev), segments=segments,
                 alpha=alpha, beta=beta, out=xd)
    assert np.array_equal(xd.cpu().numpy(), got)


def test_conv1d_k3_rejects_bad_segments(cuda_dev):
    from ncmorph_b200 import _lib, vq
    x = torch.zeros((100, 8), device=cuda_dev)
    w = torch.zeros((8, 8, 3), dtype=torch.bfloat16, device=cuda_dev)
    for segs in ([50, 49], [1] * 64 + [36], [0, 100]):   # bad sum; 65 unequal segments; empty segment
        with pytest.raises(_lib.NcmError) as ei:
            vq.conv1d_k3(x, w, None, segments=segs)
        assert ei.value.status == _lib.NCM_EINVAL


def test_post_upsample_conv_host_matches_reference_restatement(orc, cuda_dev):
    """ncm_model.apply_post_upsample_conv through the host-slice entry point.
    bf16-valued inputs: only the accumulation order differs from the reference
    restatement; arbitrary f32 inputs are rounded to bf16 for the tensor cores,
    so the bar widens to the bf16 operand rounding (2^-8 of sum |w x|)."""
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(17)
    for rows, width, exact_inputs in ((64, 32, True), (257, 96, False), (3, 8, True)):
        x = rng.standard_normal((rows, width)).astype(np.float32)
        if exact_inputs:
            x = orc.round_bf16(x)
        w = orc.round_bf16((rng.standard_normal((width, width, 3)) * 0.1).astype(np.float32))
        b = orc.round_bf16((rng.standard_normal(width) * 0.1).astype(np.float32))
        ref = orc.apply_post_upsample_conv(x, w, b)
        got = x.copy()
        ncm_model.apply_post_upsample_conv(got, w, b, rows, width)
        absprod = np.abs(x) @ (3 * np.abs(w).sum(axis=2)).T + np.abs(b) + np.abs(x)
        rel = 1e-5 if exact_inputs else 8e-3
        assert np.all(np.abs(got - ref) <= rel * absprod), (rows, width, np.abs(got - ref).max())


def test_post_upsample_conv_host_against_torch_fixture(cuda_dev):
    """The committed torch F.conv1d outputs (tests/golden/conv1d_k3.npz), with
    x and w rounded to bf16 on the device: within the bf16 operand bar."""
    from conftest import GOLDEN
    from ncmorph_b200 import ncm_model
    z = np.load(GOLDEN / "conv1d_k3.npz")
    for c in sorted(k[2:] for k in z.files if k.startswith("x_")):
        x, w, b, y = z[f"x_{c}"], z[f"w_{c}"], z[f"b_{c}"], z[f"y_{c}"]
        rows, width = x.shape
        got = x.copy()
        ncm_model.apply_post_upsample_conv(got, np.ascontiguousarray(w), b, rows, width)
        absprod = np.abs(x) @ (3 * np.abs(w).sum(axis=2)).T + np.abs(b) + np.abs(x)
        assert np.all(np.abs(got - (x + y)) <= 1e-2 * absprod), c
