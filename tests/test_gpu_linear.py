"""GPU parity of the bf16 linear (L1) against the oracle's restatement of
matmul_bf16_impl (packages/kernels/root.zig:106-142), through the C ABI.

The tensor cores accumulate in a different order from VDPBF16PS pair-FMA with
oneDNN K-blocks, so results are held to the bf16 bar (helpers.check_gemm),
not bit equality.
"""
import numpy as np
import pytest
import torch

from helpers import check_gemm, from_dev_bf16, gen_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu

SWEEP_M = [1, 64, 512, 4096, 8192]
SWEEP_KN = [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048), (2048, 128256)]


def _digest_inputs():
    T, K, N = 4, 1536, 576
    t = np.arange(T)[:, None]
    k = np.arange(K)[None, :]
    x = (((t * 29 + k * 37) % 251) - 125).astype(np.float32) / np.float32(128.0)
    n = np.arange(N)[:, None]
    w = (((n * 17 + k * 11) % 257) - 128).astype(np.float32) / np.float32(128.0)
    return x, w


def test_host_f32_entry_point_on_digest_inputs(orc, cuda_dev):
    """kernels.matmul_bf16 drop-in on the reference's digest case (root.zig:707-744)."""
    from ncmorph_b200 import kernels
    x, w = _digest_inputs()
    out = np.empty((4, 576), np.float32)
    kernels.matmul_bf16(x, w, out, 4, 1536, 576)
    ref = orc.matmul_bf16(x, w)
    check_gemm(out, ref, np.abs(x) @ np.abs(w).T, "digest case")
    # output slice holds bf16 values, as the reference's does
    assert np.array_equal(orc.round_bf16(out), out)
    same = np.mean(out.view(np.uint32) == ref.view(np.uint32))
    print(f"digest case: {same:.4f} of outputs bit-identical to the VDPBF16PS restatement")


def test_host_f32_bias_and_odd_width(orc, cuda_dev):
    from ncmorph_b200 import kernels
    rng = np.random.default_rng(3)
    T, K, N = 7, 37, 19            # K not a multiple of 8: the host entry pads with zeros
    x = rng.standard_normal((T, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.1).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    out = np.empty((T, N), np.float32)
    kernels.matmul_bf16_bias(x, w, b, out, T, K, N)
    ref = orc.matmul_bf16(x, w, b)
    xb, wb = orc.round_bf16(x), orc.round_bf16(w)
    check_gemm(out, ref, np.abs(xb) @ np.abs(wb).T + np.abs(orc.round_bf16(b)), "bias")


def test_matmul_f32_stand_in(orc, cuda_dev):
    from ncmorph_b200 import kernels
    rng = np.random.default_rng(4)
    x = rng.standard_normal((33, 64)).astype(np.float32)
    w = rng.standard_normal((34, 64)).astype(np.float32)
    out = np.empty((33, 34), np.float32)
    kernels.matmul(x, w, out, 33, 64, 34)
    xb, wb = orc.round_bf16(x).astype(np.float64), orc.round_bf16(w).astype(np.float64)
    exact = xb @ wb.T
    assert np.all(np.abs(out - exact) <= 1e-5 * (np.abs(xb) @ np.abs(wb).T) + 1e-6)


def test_reference_k_block_case_within_bar(orc, cuda_dev):
    from ncmorph_b200 import kernels
    x = np.full((1, 576), 5.960464477539063e-8, np.float32)
    x[0, 0] = 1.0
    x[0, -1] = 0.00390625
    w = np.ones((1, 576), np.float32)
    out = np.empty((1, 1), np.float32)
    kernels.matmul_bf16(x, w, out, 1, 576, 1)
    assert abs(out[0, 0] - 1.0078125) <= 2e-2 * 1.0078125


@pytest.mark.parametrize("M", SWEEP_M)
@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_llama_sweep_shapes(orc, cuda_dev, M, K, N):
    """every (M, K, N) of the Llama-3.2-1B sweep; the oracle checks sampled rows."""
    from ncmorph_b200 import kernels
    g = torch.Generator(device=cuda_dev).manual_seed(M * 7 + K + N)
    x = torch.randn((M, K), generator=g, device=cuda_dev).to(torch.bfloat16)
    w = (torch.randn((N, K), generator=g, device=cuda_dev) * 0.02).to(torch.bfloat16)
    y = kernels.linear_bf16(x, w)
    rows = np.unique(np.linspace(0, M - 1, num=min(M, 6)).astype(np.int64))
    ridx = torch.from_numpy(rows).to(cuda_dev)
    xs = orc.bf16_widen(from_dev_bf16(x[ridx]))
    wf = orc.bf16_widen(from_dev_bf16(w))
    ys = orc.bf16_widen(from_dev_bf16(y[ridx]))
    ref = orc.matmul_bf16(xs, wf, threads=8)
    check_gemm(ys, ref, np.abs(xs) @ np.abs(wf).T, f"M={M} K={K} N={N}")


@pytest.mark.parametrize("M,K,N", [(3, 64, 40), (65, 128, 300), (200, 72, 17)])
def test_bias_and_ragged_tiles(orc, cuda_dev, M, K, N):
    from ncmorph_b200 import kernels
    rng = np.random.default_rng(M + K + N)
    x = gen_bf16(rng, (M, K))
    w = gen_bf16(rng, (N, K), 0.1)
    b = gen_bf16(rng, (N,))
    y = kernels.linear_bf16(to_dev_bf16(x, cuda_dev), to_dev_bf16(w, cuda_dev), to_dev_bf16(b, cuda_dev))
    xf, wf, bf = orc.bf16_widen(x), orc.bf16_widen(w), orc.bf16_widen(b)
    ref = orc.matmul_bf16(xf, wf, bf)
    check_gemm(orc.bf16_widen(from_dev_bf16(y)), ref, np.abs(xf) @ np.abs(wf).T + np.abs(bf), "bias")


@pytest.mark.parametrize("M,K,N", [(4096, 8192, 2048),   # CTA pairs, 128 tiles: a second wave 73 % full
                                   (8192, 2048, 512),    # one-CTA 128-wide tiles
                                   (512, 2048, 512),     # 64-wide tiles, fewer tiles than SMs
                                   (4096, 2048, 3072)])  # the decoder's QKV width
def test_every_element_of_decoder_and_sweep_shapes(cuda_dev, M, K, N):
    """Every output element, bias included, against an f32 product of the
    same bf16 operands within the GEMM bar (the sweep test above checks six
    rows per shape against the oracle's bits)."""
    from ncmorph_b200 import kernels
    g = torch.Generator(device=cuda_dev).manual_seed(M + K + N)
    x = torch.randn((M, K), generator=g, device=cuda_dev).to(torch.bfloat16)
    w = (torch.randn((N, K), generator=g, device=cuda_dev) * 0.02).to(torch.bfloat16)
    b = (torch.randn((N,), generator=g, device=cuda_dev) * 0.1).to(torch.bfloat16)
    y = kernels.linear_bf16(x, w, b).float()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = x.float() @ w.float().t() + b.float()
        scale = x.float().abs() @ w.float().abs().t() + b.float().abs()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    bad = (y - ref).abs() > 2e-2 * ref.abs() + 1e-5 * scale + 1e-6
    assert int(bad.sum()) == 0, f"{int(bad.sum())} elements outside the bar, first at {bad.nonzero()[0].tolist()}"
