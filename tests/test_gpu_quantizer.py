"""GPU parity of the quantiser pieces around the RVQ levels: pre-quant
GroupNorm, the level-0 stride-4 conv cascade (tcgen05 GEMMs, bf16 operands)
and the deterministic codebook EMA, against the CPU oracle."""
import numpy as np
import pytest
import torch

from helpers import from_dev_bf16, gen_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,C,G", [(2, 1024, 384, 8), (3, 50, 24, 4), (1, 7, 8, 8)])
def test_group_norm(orc, cuda_dev, B, T, C, G):
    from ncmorph_b200 import quantizer
    x = (np.random.default_rng(B * T).standard_normal((B, T, C)) * 3 + 1).astype(np.float32)
    got = quantizer.group_norm(torch.from_numpy(x).to(cuda_dev), G).cpu().numpy()
    assert np.abs(got - orc.group_norm(x, G)).max() < 2e-5


@pytest.mark.parametrize("B,L,C", [(2, 1024, 384), (3, 64, 64), (1, 4, 8)])
def test_conv_down4_and_up4(orc, cuda_dev, B, L, C):
    from ncmorph_b200 import quantizer
    rng = np.random.default_rng(L + C)
    x = gen_bf16(rng, (B, L, C))
    w = gen_bf16(rng, (C, C, 4), 0.05)
    b = gen_bf16(rng, (C,), 0.1)
    xd, wd, bd = to_dev_bf16(x, cuda_dev), to_dev_bf16(w, cuda_dev), to_dev_bf16(b, cuda_dev)
    xf, wf, bfv = orc.bf16_widen(x), orc.bf16_widen(w), orc.bf16_widen(b)
    down = orc.bf16_widen(from_dev_bf16(quantizer.conv_down4(xd, wd, bd)))
    ref = orc.conv_down4(xf, wf, bfv)
    absprod = np.abs(xf).max() * np.abs(wf).sum(axis=(1, 2)).max() + 1
    assert np.all(np.abs(down - ref) <= 2e-2 * np.abs(ref) + 1e-5 * absprod)
    up = orc.bf16_widen(from_dev_bf16(quantizer.conv_up4(xd, wd, bd)))
    ref = orc.conv_up4(xf, wf, bfv)
    assert np.all(np.abs(up - ref) <= 2e-2 * np.abs(ref) + 1e-5 * absprod)


def test_level0_cascade_identity_init_is_mean_and_repeat(cuda_dev):
    """With the released initialisation (down: identity/4, up: identity, zero
    biases) the five-stage cascade is a mean over 1024 positions and a repeat
    back to 1024 (vq_forward_semantics.md:133-134)."""
    from ncmorph_b200 import quantizer
    C = 64
    eye = torch.eye(C, device=cuda_dev)
    wd = (eye[:, :, None].repeat(1, 1, 4) / 4).to(torch.bfloat16)
    wu = eye[:, :, None].repeat(1, 1, 4).to(torch.bfloat16)
    x = torch.randint(-8, 8, (2, 1024, C), device=cuda_dev).to(torch.bfloat16)  # exactly representable means
    z = quantizer.level0_down(x, [wd] * 5, [None] * 5)
    assert z.shape == (2, 1, C)
    assert torch.allclose(z.float()[:, 0], x.float().mean(dim=1), atol=3e-2)
    y = quantizer.level0_up(z, [wu] * 5, [None] * 5)
    assert y.shape == (2, 1024, C)
    assert torch.equal(y, z.expand(2, 1024, C))


@pytest.mark.parametrize("N,D,K", [(4096, 384, 8192), (1000, 16, 40), (1 << 16, 256, 1024)])
def test_codebook_ema_matches_oracle_and_is_deterministic(orc, cuda_dev, N, D, K):
    from ncmorph_b200 import quantizer
    rng = np.random.default_rng(N + K)
    u = rng.standard_normal((N, D)).astype(np.float32)
    codes = rng.integers(0, K, N).astype(np.int32)
    cb0 = rng.standard_normal((K, D)).astype(np.float32)
    ema = quantizer.CodebookEMA(torch.from_numpy(cb0).to(cuda_dev))
    ud, cd = torch.from_numpy(u).to(cuda_dev), torch.from_numpy(codes).to(cuda_dev)
    counts, sums = ema.stats(ud, cd)
    counts2, sums2 = ema.stats(ud, cd)
    assert torch.equal(sums, sums2)  # the same bits on every run
    cb = torch.empty((K, D), dtype=torch.float32, device=cuda_dev)
    cbb = torch.empty((K, D), dtype=torch.bfloat16, device=cuda_dev)
    ema.update(ud, cd, codebook_bf16=cbb, codebook_f32=cb)
    cnt, m, e, o_counts, o_sums = orc.ema(u, codes, np.zeros(K, np.float32), cb0, 0.99, 1e-5)
    assert np.array_equal(counts.cpu().numpy(), o_counts)
    assert np.array_equal(sums.cpu().numpy(), o_sums)  # same row order, same f32 sums
    assert np.allclose(ema.count.cpu().numpy(), cnt, rtol=1e-6)
    assert np.allclose(cb.cpu().numpy(), e, rtol=1e-5, atol=1e-5)
    assert torch.equal(cbb, cb.to(torch.bfloat16))


def test_level0_against_torch_fixture(cuda_dev):
    """tests/golden/level0.npz (torch float64 F.group_norm, F.conv1d stride 4,
    F.conv_transpose1d stride 4). The convolutions' operands are rounded to
    bf16 on the way in, so their bar is the bf16 operand rounding (2^-8 of
    sum |w x|) plus the bf16 output rounding."""
    from conftest import GOLDEN
    from ncmorph_b200 import quantizer
    z = np.load(GOLDEN / "level0.npz")
    got = quantizer.group_norm(torch.from_numpy(z["gn_x"]).to(cuda_dev), 8).cpu().numpy()
    assert np.abs(got - z["gn_y"]).max() < 2e-5
    x, w, b = (torch.from_numpy(z[k]).to(cuda_dev).to(torch.bfloat16) for k in ("conv_x", "conv_w", "conv_b"))
    absx = np.abs(z["conv_x"]).max() * np.abs(z["conv_w"]).sum(axis=(1, 2)).max() + np.abs(z["conv_b"]).max()
    for y, ref in ((quantizer.conv_down4(x, w, b), z["down_y"]), (quantizer.conv_up4(x, w, b), z["up_y"])):
        err = np.abs(y.float().cpu().numpy() - ref)
        assert np.all(err <= 1e-2 * absx + 4e-3 * np.abs(ref)), err.max()


def test_codebook_ema_rejects_out_of_range_codes(cuda_dev):
    from ncmorph_b200 import _lib, device, quantizer
    ema = quantizer.CodebookEMA(torch.zeros((16, 8), device=cuda_dev))
    u = torch.ones((40, 8), device=cuda_dev)
    codes = torch.zeros(40, dtype=torch.int32, device=cuda_dev)
    codes[7] = 16
    counts, _ = ema.stats(u, codes)
    with pytest.raises(_lib.NcmError) as ei:
        device.sync(cuda_dev)
    assert ei.value.status == _lib.NCM_ERANGE
    assert counts.sum().item() == 39  # the bad row is left out
