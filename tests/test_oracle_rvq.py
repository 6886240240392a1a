"""CPU checks of the oracle's RVQ restatement (R1-R6).

ncmorph has no RVQ code to pin against (ROADMAP.md:257-259), so these tests
anchor the restatement on the third-party semantics the spec names:
torch's F.interpolate(mode="area") for pooling (fixtures made by
tests/golden/gen_golden.py) and an exact float64 argmin with torch.argmin's
lowest-index tie rule for the distance step.
"""
import numpy as np
import pytest

from conftest import GOLDEN


def bf16_codebook(orc, rng, K, D, scale=1.0):
    return orc.bf16_bits((rng.standard_normal((K, D)) * scale).astype(np.float32))


def test_pool_matches_torch_area_interpolation(orc):
    data = np.load(GOLDEN / "pool_area.npz")
    for key in data.files:
        if not key.startswith("x_"):
            continue
        _, B, T, D, f = key.split("_")
        y = orc.pool_avg(data[key], int(f))
        ref = data["y" + key[1:]]
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), key


def test_code_sqnorm_exact(orc):
    rng = np.random.default_rng(1)
    cb = bf16_codebook(orc, rng, 33, 64)
    got = orc.code_sqnorm(cb)
    ref = (orc.bf16_widen(cb).astype(np.float64) ** 2).sum(1).astype(np.float32)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("N,D,K", [(257, 64, 300), (64, 136, 1000), (5, 8, 3)])
def test_rvq_level_is_exact_argmin_outside_near_ties(orc, N, D, K):
    rng = np.random.default_rng(N * 7 + D)
    r = rng.standard_normal((N, D)).astype(np.float32)
    cb = bf16_codebook(orc, rng, K, D)
    sq = orc.code_sqnorm(cb)
    r0 = r.copy()
    best, gap = orc.rvq_level(r, cb, sq)
    a = orc.round_bf16(r0).astype(np.float64)
    e = orc.bf16_widen(cb).astype(np.float64)
    d = (a ** 2).sum(1)[:, None] + (e ** 2).sum(1)[None, :] - 2 * a @ e.T
    exact = d.argmin(1)
    far = gap >= 1e-3
    assert np.array_equal(best[far], exact[far])
    # residual update is exact f32 subtraction of the chosen codeword
    assert np.array_equal(r, (r0 - orc.bf16_widen(cb)[best]).astype(np.float32))


def test_rvq_level_ties_pick_lowest_index(orc):
    rng = np.random.default_rng(5)
    D = 16
    base = bf16_codebook(orc, rng, 4, D)
    cb = np.concatenate([base, base[[2]], base[[1]]])  # codes 4,5 duplicate 2,1
    r = orc.bf16_widen(cb[[2, 1, 2]]).astype(np.float32).copy()
    best, gap = orc.rvq_level(r, cb, orc.code_sqnorm(cb))
    assert best.tolist() == [2, 1, 2]
    assert np.all(gap == 0)


def test_rvq_level_teacher_forcing_uses_given_codes(orc):
    rng = np.random.default_rng(9)
    r = rng.standard_normal((10, 8)).astype(np.float32)
    cb = bf16_codebook(orc, rng, 20, 8)
    forced = np.arange(10, dtype=np.int32)
    r0 = r.copy()
    best, _ = orc.rvq_level(r, cb, orc.code_sqnorm(cb), codes_in=forced)
    assert np.array_equal(r, r0 - orc.bf16_widen(cb)[forced])
    r1 = r0.copy()
    best2, _ = orc.rvq_level(r1, cb, orc.code_sqnorm(cb))
    assert np.array_equal(best, best2)


def test_threaded_level_is_bit_identical(orc):
    rng = np.random.default_rng(11)
    r = rng.standard_normal((301, 72)).astype(np.float32)
    cb = bf16_codebook(orc, rng, 130, 72)
    sq = orc.code_sqnorm(cb)
    ra, rb_ = r.copy(), r.copy()
    b1, g1 = orc.rvq_level(ra, cb, sq, threads=1)
    b4, g4 = orc.rvq_level(rb_, cb, sq, threads=4)
    assert np.array_equal(b1, b4) and np.array_equal(g1, g4) and np.array_equal(ra, rb_)


def test_decode_sums_levels_in_order(orc):
    rng = np.random.default_rng(3)
    L, K, D, N = 3, 7, 8, 5
    cbs = np.stack([bf16_codebook(orc, rng, K, D, 0.5 ** l) for l in range(L)])
    codes = rng.integers(0, K, (L, N)).astype(np.int32)
    rec = orc.rvq_decode(codes, cbs)
    e = orc.bf16_widen(cbs)
    ref = np.zeros((N, D), np.float32)
    for l in range(L):
        ref = (ref + e[l][codes[l]]).astype(np.float32)
    assert np.array_equal(rec, ref)


def test_encode_recon_error_shrinks_with_levels(orc):
    rng = np.random.default_rng(4)
    N, D, K, L = 512, 32, 64, 4
    x = orc.bf16_bits(rng.standard_normal((N, D)).astype(np.float32))
    cbs = np.stack([bf16_codebook(orc, rng, K, D, 0.5 ** l) for l in range(L)])
    best, gaps, resid, recon = orc.rvq_encode(x, cbs)
    xf = orc.bf16_widen(x)
    errs = []
    for l in range(1, L + 1):
        part = orc.rvq_decode(best[:l], cbs[:l])
        errs.append(float(((xf - part) ** 2).mean()))
    assert all(b <= a for a, b in zip(errs, errs[1:]))
    assert np.allclose(xf - recon, resid, atol=1e-5)


def test_scale_update_matches_numpy(orc):
    rng = np.random.default_rng(6)
    B, T, D, K, L, f = 2, 16, 8, 5, 3, 4
    P = B * T // f
    cbs = np.stack([bf16_codebook(orc, rng, K, D) for _ in range(L)])
    codes = rng.integers(0, K, (L, P)).astype(np.int32)
    r = rng.standard_normal((B * T, D)).astype(np.float32)
    acc = np.zeros_like(r)
    r0 = r.copy()
    orc.scale_update(codes, cbs, r, acc, B, T, f)
    q = orc.rvq_decode(codes, cbs)
    up = np.repeat(q, f, axis=0)
    assert np.array_equal(r, (r0 - up).astype(np.float32))
    assert np.array_equal(acc, up)


def test_free_running_check_accepts_near_tie_divergence_and_rejects_others(orc):
    """The free-running parity rule on planted data: a row may diverge from
    the oracle's own cascade only first at a near-tie level; a divergence
    first seen at a clear gap is a failure."""
    import pytest
    from helpers import NEAR_TIE, check_free_running
    rng = np.random.default_rng(9)
    N, D, K, L = 64, 16, 32, 4
    x = orc.bf16_bits(rng.standard_normal((N, D)).astype(np.float32))
    cbs = np.stack([bf16_codebook(orc, rng, K, D, 0.5 ** l) for l in range(L)])
    free, gaps, _, _ = orc.rvq_encode(x, cbs)
    st = check_free_running(free.copy(), free, gaps, "identical")
    assert st["diverged_rows"] == 0
    # plant a flip at level 1 of one row and pretend that level was a near-tie
    planted = free.copy()
    planted[1, 3] = (planted[1, 3] + 1) % K
    planted[2:, 3] = 0
    g = gaps.copy()
    g[1, 3] = NEAR_TIE / 2
    st = check_free_running(planted, free, g, "near-tie flip")
    assert st["diverged_rows"] == 1 and st["first_divergence_levels"] == [0, 1, 0, 0]
    # the same flip where the oracle's gap was clear must fail
    g[1, 3] = 10 * NEAR_TIE
    with pytest.raises(AssertionError):
        check_free_running(planted, free, g, "clear-gap flip")
