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

from helpers import check_codes, check_free_running, check_gemm, from_dev_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def _seeded(shape, scale, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=dev) * scale).to(torch.bfloat16)


def _threads():
    import os
    return max(1, min(64, os.cpu_count() or 1))


def run_tokenizer_case(orc, dev, B, T, Din, D, K, factors, L, sample, seed=7, free_running=False):
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
    free = []
    for s, f in enumerate(factors):
        P = N // f
        u = orc.pool_avg(r.reshape(B, T, D), f).reshape(P, D)
        cs = codes[s].cpu().numpy()
        assert cs.shape == (L, P)
        assert cs.min() >= 0 and cs.max() < K
        pr = np.sort(rng.choice(P, size=min(sample, P), replace=False))
        us = np.ascontiguousarray(u[pr])
        gaps = np.empty((L, pr.size), np.float32)
        for l in range(L):
            best, gaps[l] = orc.rvq_level(us, cbs_np[s, l], sq[s, l], codes_in=cs[l, pr], threads=_threads())
            stats.append(check_codes(cs[l, pr], best, gaps[l], f"scale {s} level {l}"))
        if free_running:
            # the scale's L levels encoded by the oracle on its own from the same pooled rows
            uf = np.ascontiguousarray(u[pr])
            fb = np.empty((L, pr.size), np.int32)
            for l in range(L):
                fb[l], _ = orc.rvq_level(uf, cbs_np[s, l], sq[s, l], threads=_threads())
            free.append(check_free_running(cs[:, pr], fb, gaps, f"scale {s}"))
        orc.scale_update(cs, cbs_np[s], r, acc, B, T, f)
    recon_bits = from_dev_bf16(recon).reshape(N, D)
    assert np.array_equal(recon_bits, orc.bf16_bits(acc))

    # L1: output projection on sampled rows
    w_out_np = orc.bf16_widen(from_dev_bf16(w_out))
    rf = orc.bf16_widen(recon_bits[rows])
    ref_y = orc.matmul_bf16(rf, w_out_np, threads=8)
    y_np = orc.bf16_widen(from_dev_bf16(y).reshape(N, Din)[rows])
    check_gemm(y_np, ref_y, np.abs(rf) @ np.abs(w_out_np).T, "output projection")
    return (stats, free) if free_running else stats


def test_tokenizer_small_all_rows(orc, cuda_dev):
    stats = run_tokenizer_case(orc, cuda_dev, B=2, T=256, Din=256, D=128, K=512, factors=[16, 8, 4, 2, 1], L=3,
                               sample=10 ** 9)
    assert sum(s["rows"] for s in stats) == 3 * (32 + 64 + 128 + 256 + 512)


def test_tokenizer_config2_full_size_sampled(orc, cuda_dev):
    """BASELINE config 2 shapes: B=8, T=2048, 2048->1024, 5 scales x 8 levels,
    K=4096; 256 pooled rows per (scale, level) teacher-forced, and the same
    rows encoded free-running by the oracle through each scale's 8 levels."""
    stats, free = run_tokenizer_case(orc, cuda_dev, B=8, T=2048, Din=2048, D=1024, K=4096, factors=[16, 8, 4, 2, 1],
                                     L=8, sample=256, free_running=True)
    print("config2 teacher-forced: flips", sum(s["flips"] for s in stats), "near-ties",
          sum(s["near_ties"] for s in stats), "of", sum(s["rows"] for s in stats), "codes")
    print("config2 free-running: rows diverged per scale", [f["diverged_rows"] for f in free], "of",
          [f["rows"] for f in free], "codes differing", [f["codes_differing"] for f in free])


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
    # oracle on a 2048-row sample: teacher-forced (every level's codes and the
    # final residual), then free-running (the oracle's own cascade of codes)
    rng = np.random.default_rng(5)
    rows = np.sort(rng.choice(N, size=2048, replace=False))
    xs = from_dev_bf16(x[torch.from_numpy(rows).to(cuda_dev)])
    cbs_np = from_dev_bf16(cbs)
    cs = codes.cpu().numpy()[:, rows]
    best, gaps, res_o, _ = orc.rvq_encode(xs, cbs_np, codes_in=cs, threads=_threads())
    st = [check_codes(cs[l], best[l], gaps[l], f"config5 level {l}") for l in range(L)]
    assert np.array_equal(resid[torch.from_numpy(rows).to(cuda_dev)].cpu().numpy(), res_o)
    free_best, _, _, _ = orc.rvq_encode(xs, cbs_np, threads=_threads())
    fr = check_free_running(cs, free_best, gaps, "config5")
    print(f"config5 teacher-forced: flips {sum(s['flips'] for s in st)}, near-ties "
          f"{sum(s['near_ties'] for s in st)} of {L * rows.size} codes; free-running: {fr['diverged_rows']} of "
          f"{rows.size} rows diverge ({fr['codes_differing']} codes), first at levels {fr['first_divergence_levels']}")


def _phi_weights(S, D, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    bound = 1.0 / np.sqrt(3 * D)   # torch's default Conv1d init scale
    w = ((torch.rand((S, D, D, 3), generator=g, device=dev) * 2 - 1) * bound).to(torch.bfloat16)
    b = (torch.rand((S, D), generator=g, device=dev) * 2 - 1) * bound
    return w, b


def run_general_case(orc, dev, B, T, Din, D, K, factors, L, mode, phi, seed=21):
    """Tokenizer with linear upsampling and/or Phi, teacher-forced like
    run_tokenizer_case. Without Phi every stage is bit-identical; with Phi
    the convolution's accumulation order differs, so the reconstruction is
    held to the north-star bar (2e-2 relative) and codes are checked on the
    oracle's own residual outside near-ties."""
    from ncmorph_b200 import kernels, vq
    S = len(factors)
    x = _seeded((B, T, Din), 1.0, dev, seed)
    w_in = _seeded((D, Din), 0.02, dev, seed + 1)
    w_out = _seeded((Din, D), 0.02, dev, seed + 2)
    decay = torch.tensor([0.6 ** l for l in range(L)], device=dev).view(1, L, 1, 1)
    cbs = (_seeded((S, L, K, D), 1.0, dev, seed + 3).float() * decay).to(torch.bfloat16)
    pw, pb = _phi_weights(S, D, dev, seed + 4) if phi else (None, None)
    codes, recon, y = vq.tokenizer_forward(x, w_in, cbs, w_out, factors, upsample=mode, phi_weight=pw, phi_bias=pb,
                                           phi_ratio=0.5)
    h = kernels.linear_bf16(x.view(B * T, Din), w_in)
    torch.cuda.synchronize()
    N = B * T
    cbs_np = from_dev_bf16(cbs)
    sq = orc.code_sqnorm(cbs_np)
    pw_np = orc.bf16_widen(from_dev_bf16(pw)) if phi else None
    pb_np = pb.cpu().numpy() if phi else None
    r = orc.bf16_widen(from_dev_bf16(h)).astype(np.float32).copy()
    acc = np.zeros_like(r)
    stats = []
    for s, f in enumerate(factors):
        P = N // f
        u = np.ascontiguousarray(orc.pool_avg(r.reshape(B, T, D), f).reshape(P, D))
        cs = codes[s].cpu().numpy()
        for l in range(L):
            best, gap = orc.rvq_level(u, cbs_np[s, l], sq[s, l], codes_in=cs[l])
            stats.append(check_codes(cs[l], best, gap, f"{mode} phi={phi} scale {s} level {l}"))
        orc.scale_update_ex(cs, cbs_np[s], r, acc, B, T, f, mode=mode,
                            phi_w=None if pw_np is None else pw_np[s], phi_b=None if pb_np is None else pb_np[s],
                            ratio=0.5)
    got = from_dev_bf16(recon).reshape(N, D)
    if not phi:
        assert np.array_equal(got, orc.bf16_bits(acc))
    else:
        g = orc.bf16_widen(got).astype(np.float64)
        ref = acc.astype(np.float64)
        rms = np.sqrt((ref ** 2).mean())
        assert np.all(np.abs(g - ref) <= 2e-2 * np.abs(ref) + 1e-3 * rms)
    # the multiscale decode of the same codes reproduces the reconstruction bit for bit
    dec = vq.multiscale_decode(codes, cbs, B, T, factors, upsample=mode, phi_weight=pw, phi_bias=pb, phi_ratio=0.5)
    assert torch.equal(dec.view(torch.int16), recon.view(torch.int16))
    return stats


@pytest.mark.parametrize("mode,phi", [("linear", False), ("nearest", True), ("linear", True)])
def test_tokenizer_upsample_modes_and_phi(orc, cuda_dev, mode, phi):
    stats = run_general_case(orc, cuda_dev, B=2, T=256, Din=256, D=128, K=512, factors=[16, 8, 4, 2, 1], L=3,
                             mode=mode, phi=phi)
    print(mode, phi, "flips", sum(s["flips"] for s in stats), "near", sum(s["near_ties"] for s in stats))


def test_multiscale_decode_nearest_matches_tokenizer(cuda_dev):
    """Default mode (nearest, no Phi) at config-2 shapes: decode(codes) == recon."""
    from ncmorph_b200 import vq
    B, T, Din, D, K, L, factors = 8, 2048, 2048, 1024, 4096, 8, [16, 8, 4, 2, 1]
    x = _seeded((B, T, Din), 1.0, cuda_dev, 31)
    w_in = _seeded((D, Din), 0.02, cuda_dev, 32)
    w_out = _seeded((Din, D), 0.02, cuda_dev, 33)
    cbs = _seeded((len(factors), L, K, D), 0.5, cuda_dev, 34)
    for mode in ("nearest", "linear"):
        codes, recon, _ = vq.tokenizer_forward(x, w_in, cbs, w_out, factors, upsample=mode)
        dec = vq.multiscale_decode(codes, cbs, B, T, factors, upsample=mode)
        assert torch.equal(dec.view(torch.int16), recon.view(torch.int16)), mode


def test_tokenizer_config2_phi_linear_properties(cuda_dev):
    """Config-2 shapes with linear upsampling and Phi at every scale: codes in
    range, decode == recon, and recon equal to the sum over scales of
    Phi(up(q_s)) recomputed through the separate upsample and conv entry points."""
    from ncmorph_b200 import vq
    B, T, Din, D, K, L, factors = 8, 2048, 2048, 1024, 4096, 8, [16, 8, 4, 2, 1]
    S = len(factors)
    x = _seeded((B, T, Din), 1.0, cuda_dev, 41)
    w_in = _seeded((D, Din), 0.02, cuda_dev, 42)
    w_out = _seeded((Din, D), 0.02, cuda_dev, 43)
    decay = torch.tensor([0.6 ** l for l in range(L)], device=cuda_dev).view(1, L, 1, 1)
    cbs = (_seeded((S, L, K, D), 1.0, cuda_dev, 44).float() * decay).to(torch.bfloat16)
    pw, pb = _phi_weights(S, D, cuda_dev, 45)
    codes, recon, y = vq.tokenizer_forward(x, w_in, cbs, w_out, factors, upsample="linear", phi_weight=pw,
                                           phi_bias=pb, phi_ratio=0.5)
    for c in codes:
        assert int(c.min()) >= 0 and int(c.max()) < K
    dec = vq.multiscale_decode(codes, cbs, B, T, factors, upsample="linear", phi_weight=pw, phi_bias=pb)
    assert torch.equal(dec.view(torch.int16), recon.view(torch.int16))
    acc = torch.zeros((B * T, D), device=cuda_dev)
    for s, f in enumerate(factors):
        q = torch.zeros((B * T // f, D), device=cuda_dev)
        for l in range(L):
            q += cbs[s, l].float()[codes[s][l].long()]
        Q = vq.upsample(q.view(B, T // f, D), T, "linear").view(B * T, D)
        acc += vq.conv1d_k3(Q, pw[s], pb[s], segments=[T] * B, alpha=0.5, beta=0.5)
    assert torch.equal(acc.to(torch.bfloat16).view(torch.int16), recon.view(B * T, D).view(torch.int16))


def test_streamed_inputs_are_read_after_their_copy(cuda_dev):
    """Inputs copied in on a second stream (two device buffers; three host
    inputs cycle, so a buffer holds a different input at each use) and
    consumed after a cross-stream event wait: every step's codes equal the
    codes of its own input computed directly.
    The kernels launch with programmatic stream serialization, which must not
    let a kernel run ahead of an event the stream waits on."""
    from ncmorph_b200 import vq
    B, T, Din, D, K, L = 2, 256, 256, 128, 256, 2
    factors = [4, 2, 1]
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    xs = [torch.randn((B, T, Din), generator=g, device=cuda_dev).to(torch.bfloat16) for _ in range(3)]
    w_in = (torch.randn((D, Din), generator=g, device=cuda_dev) * 0.05).to(torch.bfloat16)
    w_out = (torch.randn((Din, D), generator=g, device=cuda_dev) * 0.05).to(torch.bfloat16)
    cbs = torch.randn((len(factors), L, K, D), generator=g, device=cuda_dev).to(torch.bfloat16)
    direct = [torch.cat([c.reshape(-1) for c in vq.tokenizer_forward(x, w_in, cbs, w_out, factors)[0]]) for x in xs]
    hosts = [x.cpu().pin_memory() for x in xs]
    cur, cp = torch.cuda.current_stream(), torch.cuda.Stream(device=cuda_dev)
    bufs = [torch.empty_like(xs[0]), torch.empty_like(xs[0])]
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]
    outs = []
    steps = 8
    with torch.cuda.stream(cp):
        cp.wait_stream(cur)
        bufs[0].copy_(hosts[0], non_blocking=True)
        copied[0].record(cp)
    for i in range(steps):
        b = i & 1
        if i + 1 < steps:
            with torch.cuda.stream(cp):
                if i >= 1:
                    cp.wait_event(consumed[b ^ 1])
                bufs[b ^ 1].copy_(hosts[(i + 1) % 3], non_blocking=True)
                copied[b ^ 1].record(cp)
        cur.wait_event(copied[b])
        codes = vq.tokenizer_forward(bufs[b], w_in, cbs, w_out, factors)[0]
        consumed[b].record(cur)
        outs.append(torch.cat([c.reshape(-1) for c in codes]))
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(o, direct[i % 3]), i
