"""GPU parity of the multiscale tokenizer forward (R4-R6, with the L1 input and
output projections), and of the full-size RVQ configurations, against the
CPU oracle through the C ABI.

The oracle is teacher-forced at the stage boundaries: it starts from the
GPU's input projection h (itself checked against the oracle linear), and at
each scale advances with the GPU's codes. Pooling, the scale updates and the
reconstruction are then bit-identical on both sides; codes must agree
outside near-ties; the output projection is held to the bf16 GEMM bar.
"""
import numpy as np
import pytest
import torch

from helpers import check_codes, check_gemm, from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def _seeded(shape, scale, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=dev) * scale).to(torch.bfloat16)


def run_tokenizer_case(orc, dev, B, T, Din, D, K, factors, L, sample, seed=7):
    from ncmorph_b200 import kernels, vq
    S = len(factors)
    x = _seeded((B, T, Din), 1.0, dev, seed)
    w_in = _seeded((D, Din), 0.02, dev, seed + 1)
    w_out = _seeded((Din, D), 0.02, dev, seed + 2)
    decay = torch.tensor([0.6 ** l for l in range(L)], device=dev).view(1, L, 1, 1)
    cbs = (_seeded((S, L, K, D), 1.0, dev, seed + 3).float() * decay).to(torch.bfloat16)
    codes, recon, y = vq.tokenizer_forward(x, w_in, cbs, w_out, factors)
    h = kernels.linear_bf16(x.view(B * T, Din), w_in)
    torch.cuda.synchronize()

    rng = np.random.default_rng(seed)
    N = B * T
    x_np = from_dev_bf16(x).reshape(N, Din)
    w_in_np = from_dev_bf16(w_in)
    h_bits = from_dev_bf16(h)
    cbs_np = from_dev_bf16(cbs)
    sq = orc.code_sqnorm(cbs_np)

    # L1: input projection on sampled rows
    rows = np.sort(rng.choice(N, size=min(sample, N), replace=False))
    xf = orc.bf16_widen(x_np[rows])
    wf = orc.bf16_widen(w_in_np)
    ref_h = orc.matmul_bf16(xf, wf, threads=8)
    check_gemm(orc.bf16_widen(h_bits[rows]), ref_h, np.abs(xf) @ np.abs(wf).T, "input projection")

    # R4-R6 teacher-forced from the GPU's h
    r = orc.bf16_widen(h_bits).astype(np.float32).copy()
    acc = np.zeros_like(r)
    stats = []
    for s, f in enumerate(factors):
        P = N // f
        u = orc.pool_avg(r.reshape(B, T, D), f).reshape(P, D)
        cs = codes[s].cpu().numpy()
        assert cs.shape == (L, P)
        assert cs.min() >= 0 and cs.max() < K
        pr = np.sort(rng.choice(P, size=min(sample, P), replace=False))
        us = np.ascontiguousarray(u[pr])
        for l in range(L):
            best, gap = orc.rvq_level(us, cbs_np[s, l], sq[s, l], codes_in=cs[l, pr])
            stats.append(check_codes(cs[l, pr], best, gap, f"scale {s} level {l}"))
        orc.scale_update(cs, cbs_np[s], r, acc, B, T, f)
    recon_bits = from_dev_bf16(recon).reshape(N, D)
    assert np.array_equal(recon_bits, orc.bf16_bits(acc))

    # L1: output projection on sampled rows
    w_out_np = orc.bf16_widen(from_dev_bf16(w_out))
    rf = orc.bf16_widen(recon_bits[rows])
    ref_y = orc.matmul_bf16(rf, w_out_np, threads=8)
    y_np = orc.bf16_widen(from_dev_bf16(y).reshape(N, Din)[rows])
    check_gemm(y_np, ref_y, np.abs(rf) @ np.abs(w_out_np).T, "output projection")
    return stats


def test_tokenizer_small_all_rows(orc, cuda_dev):
    stats = run_tokenizer_case(orc, cuda_dev, B=2, T=256, Din=256, D=128, K=512, factors=[16, 8, 4, 2, 1], L=3,
                               sample=10 ** 9)
    assert sum(s["rows"] for s in stats) == 3 * (32 + 64 + 128 + 256 + 512)


def test_tokenizer_config2_full_size_sampled(orc, cuda_dev):
    """BASELINE config 2 shapes: B=8, T=2048, 2048->1024, 5 scales x 8 levels, K=4096."""
    stats = run_tokenizer_case(orc, cuda_dev, B=8, T=2048, Din=2048, D=1024, K=4096, factors=[16, 8, 4, 2, 1],
                               L=8, sample=48)
    print("config2 flips", sum(s["flips"] for s in stats), "near", sum(s["near_ties"] for s in stats))


def test_config5_encode_sampled(orc, cuda_dev):
    """BASELINE config 5 at full size: N=2^20, D=1024, 8 levels x K=16384, level l ~ N(0, 0.6^l).
    Oracle on a row sample (teacher-forced); size-independent properties on all rows."""
    from ncmorph_b200 import vq
    N, D, K, L = 1 << 20, 1024, 16384, 8
    x = _seeded((N, D), 1.0, cuda_dev, 11)
    decay = torch.tensor([0.6 ** l for l in range(L)], device=cuda_dev).view(L, 1, 1)
    cbs = (_seeded((L, K, D), 1.0, cuda_dev, 12).float() * decay).to(torch.bfloat16)
    codes, recon, resid = vq.rvq_encode(x, cbs, want_residual=True)
    torch.cuda.synchronize()
    # properties over every row
    assert int(codes.min()) >= 0 and int(codes.max()) < K
    # x = recon + residual up to the bf16 rounding of recon (f32 sums of the same codewords)
    rec_f32 = torch.zeros((N, D), device=cuda_dev)
    for l in range(L):
        rec_f32 += cbs[l].float()[codes[l].long()]
    assert torch.equal(rec_f32.to(torch.bfloat16).view(torch.int16), recon.view(torch.int16))
    err = (x.float() - rec_f32 - resid).abs().max().item()
    assert err < 1e-4, err
    # on every row and level the chosen code is at least as near as 8 random
    # other codes (the synthetic codebooks are too spread for the residual to
    # shrink at every level, so nearness, not shrinkage, is the property)
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    r = x.float()
    for l in range(L):
        a = r.to(torch.bfloat16).float()
        e = cbs[l].float()
        d_best = ((a - e[codes[l].long()]) ** 2).sum(1)
        for _ in range(8):
            j = torch.randint(0, K, (N,), generator=g, device=cuda_dev)
            d_j = ((a - e[j]) ** 2).sum(1)
            assert bool((d_best <= d_j * (1 + 1e-3)).all()), f"level {l}: a random code beats the chosen one"
        r = r - e[codes[l].long()]
        del a, e, d_best
    del r, rec_f32
    # oracle, teacher-forced, on a row sample
    rng = np.random.default_rng(5)
    rows = np.sort(rng.choice(N, size=24, replace=False))
    xs = from_dev_bf16(x[torch.from_numpy(rows).to(cuda_dev)])
    cbs_np = from_dev_bf16(cbs)
    cs = codes.cpu().numpy()[:, rows]
    best, gaps, res_o, _ = orc.rvq_encode(xs, cbs_np, codes_in=cs, threads=8)
    for l in range(L):
        check_codes(cs[l], best[l], gaps[l], f"config5 level {l}")
    assert np.array_equal(resid[torch.from_numpy(rows).to(cuda_dev)].cpu().numpy(), res_o)
