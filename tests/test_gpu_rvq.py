"""GPU parity of the RVQ path (R1-R6) against the CPU oracle, through the C ABI.

Codes are checked level by level with teacher forcing: the oracle advances
its residual with the GPU's codes, so both sides see bit-identical inputs at
every level and any code difference is a genuine argmin difference (allowed
only at near-ties, which are counted).
"""
import numpy as np
import pytest
import torch

from helpers import check_codes, from_dev_bf16, gen_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def _cbs(rng, L, K, D, decay):
    return np.stack([gen_bf16(rng, (K, D), decay ** l) for l in range(L)])


def test_code_sqnorm_bit_exact(orc, cuda_dev):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(0)
    cb = gen_bf16(rng, (3, 1000, 136))
    got = vq.code_sqnorm(to_dev_bf16(cb, cuda_dev)).cpu().numpy()
    assert np.array_equal(got, orc.code_sqnorm(cb))


@pytest.mark.parametrize("N,D,K", [
    (4096, 256, 1024),   # config 1 shape, one level
    (1000, 136, 700),    # ragged rows, D not a multiple of 64, K not a multiple of 256
    (300, 64, 5000),     # few rows, many codes: code-split path
    (1, 8, 1),           # smallest legal problem
    (129, 1024, 257),    # one row past a 128-row block, one code past a 256-code tile
])
def test_rvq_level_matches_oracle(orc, cuda_dev, N, D, K):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(N + D + K)
    r = rng.standard_normal((N, D)).astype(np.float32)
    cb = gen_bf16(rng, (K, D))
    sq = orc.code_sqnorm(cb)
    rd = torch.from_numpy(r).to(cuda_dev)
    codes = vq.rvq_level(rd, to_dev_bf16(cb, cuda_dev), torch.from_numpy(sq).to(cuda_dev)).cpu().numpy()
    r_orc = r.copy()
    best, gap = orc.rvq_level(r_orc, cb, sq, codes_in=codes)
    check_codes(codes, best, gap, f"level N={N} D={D} K={K}")
    assert np.array_equal(rd.cpu().numpy(), r_orc)  # f32 residual update, bit for bit


def test_rvq_level_ties_pick_lowest_index(cuda_dev, orc):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(5)
    D = 64
    base = gen_bf16(rng, (300, D))
    cb = np.concatenate([base, base[[7]], base[[299]]])   # 300 == 7 and 301 == 299, across code tiles
    r = orc.bf16_widen(cb[[7, 299, 7]]).astype(np.float32).copy()
    codes = vq.rvq_level(torch.from_numpy(r).to(cuda_dev), to_dev_bf16(cb, cuda_dev)).cpu().numpy()
    assert codes.tolist() == [7, 299, 7]


def test_config1_encode_decode(orc, cuda_dev):
    """N=4096, D=256, 4 levels of K=1024, level l ~ N(0, 0.5^l)."""
    from ncmorph_b200 import vq
    rng = np.random.default_rng(20260)
    N, D, K, L = 4096, 256, 1024, 4
    x = gen_bf16(rng, (N, D))
    cbs = _cbs(rng, L, K, D, 0.5)
    codes_d, recon_d, resid_d = vq.rvq_encode(to_dev_bf16(x, cuda_dev), to_dev_bf16(cbs, cuda_dev),
                                              want_residual=True)
    codes = codes_d.cpu().numpy()
    best, gaps, resid, recon = orc.rvq_encode(x, cbs, codes_in=codes)
    stats = [check_codes(codes[l], best[l], gaps[l], f"level {l}") for l in range(L)]
    flips = sum(s["flips"] for s in stats)
    print(f"config1 flips={flips} near_ties={sum(s['near_ties'] for s in stats)} of {N * L}")
    assert np.array_equal(resid_d.cpu().numpy(), resid)
    assert np.array_equal(from_dev_bf16(recon_d), orc.bf16_bits(recon))
    # decode entry point reproduces the encode's reconstruction
    assert torch.equal(vq.rvq_decode(codes_d, to_dev_bf16(cbs, cuda_dev)).view(torch.int16),
                       recon_d.view(torch.int16))
    # free-running oracle agrees on every row without a near-tie at any level
    fb, fg, _, frecon = orc.rvq_encode(x, cbs)
    clean = (fg >= 1e-3).all(axis=0)
    assert np.array_equal(codes[:, clean], fb[:, clean])
    assert clean.mean() > 0.5


@pytest.mark.parametrize("N,D,K,L,keep", [
    (148 * 128 + 37, 256, 512, 3, True),
    (148 * 128 + 37, 256, 512, 3, False),   # the last level decodes without updating
    (300 * 128, 64, 300, 2, True),
    (300 * 128, 64, 300, 1, False),         # one level: its input is the bf16 rows themselves
    (160 * 128, 72, 32, 37, False),         # two 32-level code groups in the decode
    (60 * 256 + 77, 256, 1024, 2, True),    # 61 ragged 256-row units: CTA pairs with some pairs idle-free
])
def test_fused_update_path_matches_oracle(orc, cuda_dev, N, D, K, L, keep):
    """Row blocks >= SM count: one code split, so the residual update (f32 and
    its bf16 shadow) runs inside the distance kernel; the last level updates
    only when the residual is kept."""
    from ncmorph_b200 import vq
    rng = np.random.default_rng(N + K + L)
    x = gen_bf16(rng, (N, D))
    cbs = _cbs(rng, L, K, D, 0.5 if L < 8 else 0.8)
    cbs_d = to_dev_bf16(cbs, cuda_dev)
    codes_d, recon_d, resid_d = vq.rvq_encode(to_dev_bf16(x, cuda_dev), cbs_d, want_residual=keep)
    codes = codes_d.cpu().numpy()
    best, gaps, resid, recon = orc.rvq_encode(x, cbs, codes_in=codes)
    for l in range(L):
        check_codes(codes[l], best[l], gaps[l], f"fused level {l}")
    if keep:
        assert np.array_equal(resid_d.cpu().numpy(), resid)
    assert np.array_equal(from_dev_bf16(recon_d), orc.bf16_bits(recon))
    # the decode entry point reproduces the encode's reconstruction
    assert torch.equal(vq.rvq_decode(codes_d, cbs_d).view(torch.int16), recon_d.view(torch.int16))
    if L > 3:
        return
    # single-level entry point on the same rows (f32 residual in, no shadow out)
    r = orc.bf16_widen(x).astype(np.float32).copy()
    rd = torch.from_numpy(r).to(cuda_dev)
    c0 = vq.rvq_level(rd, to_dev_bf16(cbs[0], cuda_dev)).cpu().numpy()
    b0, g0 = orc.rvq_level(r, cbs[0], orc.code_sqnorm(cbs[0]), codes_in=c0)
    check_codes(c0, b0, g0, "fused single level")
    assert np.array_equal(rd.cpu().numpy(), r)


@pytest.mark.parametrize("pinned", [True, False])
def test_host_pipelined_encode_matches_device_encode(cuda_dev, pinned):
    """ncm_rvq_encode_host over several row chunks equals ncm_rvq_encode bit for bit."""
    from ncmorph_b200 import vq
    N, D, K, L = 300_000, 64, 256, 2   # > 2 chunks of ~7 waves of 128-row blocks
    g = torch.Generator(device=cuda_dev).manual_seed(4)
    x = torch.randn((N, D), generator=g, device=cuda_dev).to(torch.bfloat16)
    cbs = (torch.randn((L, K, D), generator=g, device=cuda_dev)).to(torch.bfloat16)
    codes_d, recon_d, _ = vq.rvq_encode(x, cbs)
    x_host = x.cpu()
    if pinned:
        x_host = x_host.pin_memory()
    codes_h, recon_h = vq.rvq_encode_host(x_host, cbs)
    assert torch.equal(codes_h, codes_d.cpu())
    assert torch.equal(recon_h.view(torch.int16), recon_d.cpu().view(torch.int16))
    codes_only, none = vq.rvq_encode_host(x_host, cbs, want_recon=False)
    assert none is None and torch.equal(codes_only, codes_d.cpu())


@pytest.mark.parametrize("N,L,D,K", [
    (333, 8, 1024, 4096),   # the encode's shape class: one 8-level gather group, 4 column chunks
    (100, 40, 264, 50),     # two 32-level code groups, 5 levels past a multiple of 8, a ragged last chunk
    (17, 3, 8, 5),          # one active lane, fewer levels than a gather group
    (9, 64, 520, 7),        # the most levels an encode takes
])
def test_decode_bit_exact(orc, cuda_dev, N, L, D, K):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(N * L + D)
    cbs = np.stack([gen_bf16(rng, (K, D), 0.7 ** l) for l in range(L)])
    codes = rng.integers(0, K, (L, N), dtype=np.int32)
    got = vq.rvq_decode(torch.from_numpy(codes).to(cuda_dev), to_dev_bf16(cbs, cuda_dev))
    assert np.array_equal(from_dev_bf16(got), orc.bf16_bits(orc.rvq_decode(codes, cbs)))


def test_decode_skips_only_rows_with_a_bad_code(orc, cuda_dev):
    from ncmorph_b200 import _lib, device, vq
    rng = np.random.default_rng(11)
    L, N, D, K = 36, 20, 136, 30
    cbs = np.stack([gen_bf16(rng, (K, D)) for _ in range(L)])
    codes = rng.integers(0, K, (L, N), dtype=np.int32)
    codes[33, 4] = K        # a bad code in the second 32-level group
    codes[0, 9] = -1
    out = torch.full((N, D), 7, dtype=torch.int16, device=cuda_dev).view(torch.bfloat16)
    vq.rvq_decode(torch.from_numpy(codes).to(cuda_dev), to_dev_bf16(cbs, cuda_dev), recon=out)
    with pytest.raises(_lib.NcmError) as ei:
        device.sync(cuda_dev)
    assert ei.value.status == _lib.NCM_ERANGE
    got = from_dev_bf16(out)
    good = [n for n in range(N) if n not in (4, 9)]
    assert np.array_equal(got[good], orc.bf16_bits(orc.rvq_decode(codes[:, good], cbs)))
    assert (got[[4, 9]] == 7).all()   # left as they were


def test_decode_rejects_out_of_range_codes(cuda_dev):
    from ncmorph_b200 import _lib, device, vq
    cbs = torch.zeros((2, 16, 8), dtype=torch.bfloat16, device=cuda_dev)
    codes = torch.zeros((2, 4), dtype=torch.int32, device=cuda_dev)
    codes[1, 2] = 16
    vq.rvq_decode(codes, cbs)
    with pytest.raises(_lib.NcmError) as ei:
        device.sync(cuda_dev)
    assert ei.value.status == _lib.NCM_ERANGE
    device.sync(cuda_dev)  # the error word was cleared; the context stays usable


@pytest.mark.parametrize("B,T,D,f", [(2, 64, 24, 16), (3, 32, 1024, 2), (1, 8, 8, 1), (8, 2048, 64, 4)])
def test_pool_bit_exact(orc, cuda_dev, B, T, D, f):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(B * T + D)
    x = rng.standard_normal((B, T, D)).astype(np.float32)
    y = vq.pool_avg(torch.from_numpy(x).to(cuda_dev), f).cpu().numpy()
    assert np.array_equal(y.view(np.uint32), orc.pool_avg(x, f).view(np.uint32))


def test_argument_validation(cuda_dev):
    from ncmorph_b200 import _lib, vq
    r = torch.zeros((4, 12), device=cuda_dev)            # D=12 is not a multiple of 8
    cb = torch.zeros((3, 12), dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(_lib.NcmError) as ei:
        vq.rvq_level(r, cb)
    assert ei.value.status == _lib.NCM_EINVAL


@pytest.mark.parametrize("N,D,K", [(300, 64, 5000), (148 * 128 + 37, 128, 512), (1000, 136, 700)])
def test_rvq_level_top2_gap_matches_oracle(orc, cuda_dev, N, D, K):
    """Top-2 gap output (code-split and fused plans): the same codes and residual
    as ncm_rvq_level, and the oracle's relative gap within accumulation noise."""
    from ncmorph_b200 import vq
    rng = np.random.default_rng(N + 3 * K)
    r = rng.standard_normal((N, D)).astype(np.float32)
    cb = gen_bf16(rng, (K, D))
    cbd = to_dev_bf16(cb, cuda_dev)
    r1 = torch.from_numpy(r).to(cuda_dev)
    r2 = r1.clone()
    codes, gap = vq.rvq_level_top2(r1, cbd)
    plain = vq.rvq_level(r2, cbd)
    assert torch.equal(codes, plain) and torch.equal(r1, r2)
    r_orc = r.copy()
    best, ogap = orc.rvq_level(r_orc, cb, orc.code_sqnorm(cb), codes_in=codes.cpu().numpy())
    g = gap.cpu().numpy()
    assert np.all(g >= 0)
    assert np.abs(g - ogap).max() <= 1e-4, np.abs(g - ogap).max()


def test_rvq_level_top2_duplicate_codeword_gap_is_zero(cuda_dev):
    from ncmorph_b200 import vq
    rng = np.random.default_rng(6)
    base = gen_bf16(rng, (300, 64))
    cb = np.concatenate([base, base[[7]]])
    from oracle import pyoracle as orc
    r = orc.bf16_widen(base[[7, 7, 3]]).astype(np.float32).copy()
    codes, gap = vq.rvq_level_top2(torch.from_numpy(r).to(cuda_dev), to_dev_bf16(cb, cuda_dev))
    assert codes.tolist()[:2] == [7, 7]
    assert gap.tolist()[:2] == [0.0, 0.0] and gap.tolist()[2] > 0


@pytest.mark.parametrize("N,D,K,L,keep", [
    (4096, 256, 1024, 4, True),      # 32 row blocks x clusters of 4 CTAs
    (4096, 256, 1024, 4, False),
    (1000, 136, 700, 3, True),       # ragged rows, columns (slices of 48 and 40) and codes
    (2048, 1024, 2048, 8, False),    # D = 1024 (slices of 128 columns: residual in global memory)
    (640, 64, 300, 6, True),         # 5 row blocks, slice 32 over two CTAs
    (4096, 256, 256, 5, True),       # one code tile: clusters of one CTA
    # the operand kept in shared memory (64-column slices, D <= 256): clusters of 2 and 3 CTAs,
    # a ragged last slice (56 columns) and ragged rows
    (2000, 128, 512, 5, True),
    (1536, 192, 768, 4, False),
    (3000, 248, 1024, 4, True),
])
def test_small_encode_in_one_launch_matches_levels(orc, cuda_dev, N, D, K, L, keep):
    """Few row blocks: every level runs in one launch, one cluster of CTAs per
    128-row block sharing the code range through distributed shared memory.
    Codes and residual must equal ncm_rvq_level applied level by level (the
    split plan with rvq_apply_kernel) bit for bit, and the oracle outside
    near-ties; the reconstruction equals the oracle's."""
    from ncmorph_b200 import vq
    rng = np.random.default_rng(N * 3 + D + K + L)
    x = gen_bf16(rng, (N, D))
    cbs = _cbs(rng, L, K, D, 0.6)
    xd, cbs_d = to_dev_bf16(x, cuda_dev), to_dev_bf16(cbs, cuda_dev)
    codes_d, recon_d, resid_d = vq.rvq_encode(xd, cbs_d, want_residual=keep)
    # level by level through the single-level entry point
    r = xd.float().clone()
    ref_codes = torch.stack([vq.rvq_level(r, cbs_d[l]) for l in range(L)])
    torch.cuda.synchronize()
    assert torch.equal(codes_d, ref_codes)
    if keep:
        assert torch.equal(resid_d, r)
    codes = codes_d.cpu().numpy()
    best, gaps, resid, recon = orc.rvq_encode(x, cbs, codes_in=codes)
    for l in range(L):
        check_codes(codes[l], best[l], gaps[l], f"one-launch level {l}")
    if keep:
        assert np.array_equal(resid_d.cpu().numpy(), resid)
    assert np.array_equal(from_dev_bf16(recon_d), orc.bf16_bits(recon))
