"""Pins the CPU oracle to ncmorph's own golden vectors and known-answer tests.

Every constant below is taken from the reference's tests (cited per test);
the oracle must reproduce each one bit-exactly before it is trusted as the
parity checker for the GPU kernels.
"""
import numpy as np
import pytest

from conftest import GOLDEN


def _pairs():
    rows = [l.split() for l in (GOLDEN / "bf16_pairs.txt").read_text().splitlines() if not l.startswith("#")]
    a = np.array([int(r[0], 16) for r in rows], dtype=np.uint32)
    b = np.array([int(r[1], 16) for r in rows], dtype=np.uint16)
    return a, b


def test_bf16_matches_every_pytorch_vector(orc):
    # packages/bf16/root.zig:43-48 over packages/bf16/vectors.zig
    a, b = _pairs()
    assert a.size == 4119
    got = orc.bf16_bits(a.view(np.float32))
    bad = np.nonzero(got != b)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first f32 bits {a[bad[0]]:08X}"


def test_bf16_round_trips_every_pattern(orc):
    # packages/bf16/root.zig:50-59
    bits = np.arange(0x10000, dtype=np.uint32).astype(np.uint16)
    back = orc.bf16_bits(orc.bf16_widen(bits))
    is_nan = (bits & 0x7FFF) > 0x7F80
    expected = np.where(is_nan, np.uint16(0x7FC0), bits)
    assert np.array_equal(back, expected)


def _digest_inputs():
    T, K, N = 4, 1536, 576
    t = np.arange(T)[:, None]
    k = np.arange(K)[None, :]
    x = (((t * 29 + k * 37) % 251) - 125).astype(np.float32) / np.float32(128.0)
    n = np.arange(N)[:, None]
    w = (((n * 17 + k * 11) % 257) - 128).astype(np.float32) / np.float32(128.0)
    return x, w


def fnv1a_bf16(values: np.ndarray) -> int:
    digest = 14695981039346656037
    for v in values.astype(np.float32).ravel().view(np.uint32):
        digest = ((digest ^ int(v >> 16)) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return digest


def test_bf16_linear_digest(orc):
    # packages/kernels/root.zig:707-744 (M=4, K=1536 -> 1024+512 blocks, N=576)
    x, w = _digest_inputs()
    out = orc.matmul_bf16(x, w)
    assert fnv1a_bf16(out) == 0x547F69F667C8103F
    flat = out.ravel()
    assert flat[0] == np.float32(-0.466796875)
    assert flat[1] == np.float32(1.109375)
    assert flat[1793] == np.float32(-0.796875)


def test_bf16_linear_digest_threaded_same_bits(orc):
    x, w = _digest_inputs()
    assert np.array_equal(orc.matmul_bf16(x, w, threads=4).view(np.uint32), orc.matmul_bf16(x, w).view(np.uint32))


def test_bf16_linear_flushes_subnormal_products(orc):
    # packages/kernels/root.zig:746-755
    v = np.float32(5.421010862427522e-20)
    out = orc.matmul_bf16(np.array([[v, v]], np.float32), np.array([[v, v]], np.float32))
    assert out[0, 0] == 0.0


def test_bf16_linear_combines_512_wide_k_blocks(orc):
    # packages/kernels/root.zig:757-770
    x = np.full((1, 576), 5.960464477539063e-8, np.float32)
    x[0, 0] = 1.0
    x[0, -1] = 0.00390625
    w = np.ones((1, 576), np.float32)
    assert orc.matmul_bf16(x, w)[0, 0] == np.float32(1.0078125)


def test_matmul_hand_computed(orc):
    # packages/kernels/root.zig:676-688
    x = np.array([[5, 6], [7, 8]], np.float32)
    w = np.array([[1, 2], [3, 4]], np.float32)
    assert np.array_equal(orc.matmul(x, w).ravel(), np.array([17, 39, 23, 53], np.float32))


@pytest.mark.parametrize("T,K,N", [(1, 35, 4), (3, 7, 5), (2, 1, 3), (33, 35, 34)])
def test_matmul_blocked_equals_reference_and_d53(orc, T, K, N):
    # packages/kernels/root.zig:690-705, check_random_case :836-872
    rng = np.random.default_rng(0xB12026 + T * 1000 + K)
    x = (rng.random((T, K), dtype=np.float32) * 2 - 1).astype(np.float32)
    w = (rng.random((N, K), dtype=np.float32) * 2 - 1).astype(np.float32)
    blocked = orc.matmul(x, w)
    ref = orc.matmul(x, w, reference=True)
    assert np.array_equal(blocked.view(np.uint32), ref.view(np.uint32))
    exact = x.astype(np.float64) @ w.astype(np.float64).T
    absprod = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    assert np.all(np.abs(blocked - exact) <= (K + 1) * 2.0 ** -24 * absprod)


def test_rms_norm_cascade_sum_bits(orc):
    # packages/kernels/root.zig:799-817
    x = ((np.arange(896) * 17) % 101 + 1).astype(np.float32) * np.float32(0.125)
    assert np.float32(orc.sum_squares_pinned(x)).view(np.uint32) == 0x473BE6E0
    t = (np.arange(11) + 1).astype(np.float32) * np.float32(0.125)
    assert np.float32(orc.sum_squares_pinned(t)).view(np.uint32) == 0x40FD0000


def test_head_sum_of_squares_order(orc):
    """The order the QK-norm kernel sums one 64-wide head in: the cascade of
    root.zig:152-224 with two 4x8 accumulator rows and no full level step,
    acc[r][l] = x[8r+l]^2 + x[8(r+4)+l]^2, vs[l] = ((acc0 + acc1) + acc2) + acc3,
    sum = vs[0] + ... + vs[7], each step rounded to f32."""
    rng = np.random.default_rng(12)
    f = np.float32
    for scale in (1.0, 1e-3, 300.0):
        for _ in range(200):
            x = (rng.standard_normal(64) * scale).astype(f)
            sq = (x * x).astype(f).reshape(8, 8)
            acc = [f(sq[r] + sq[r + 4]) for r in range(4)]
            vs = f(f(f(acc[0] + acc[1]) + acc[2]) + acc[3])
            total = f(0)
            for v in vs:
                total = f(total + v)
            assert total.view(np.uint32) == np.float32(orc.sum_squares_pinned(x)).view(np.uint32)


def test_small_exact_cases(orc):
    # packages/kernels/root.zig:772-797
    assert np.array_equal(orc.softmax(np.array([2, 2], np.float32)), np.array([0.5, 0.5], np.float32))
    assert orc.silu(np.array([0.0], np.float32))[0] == 0.0
    out = orc.rms_norm(np.full(4, 3, np.float32), np.ones(4, np.float32), 0.0)
    assert np.array_equal(out, np.ones(4, np.float32))


def test_elementwise_d53_bounds(orc):
    # packages/kernels/root.zig:828-923 (D53 bounds, seeded inputs)
    rng = np.random.default_rng(0xB22026)
    x = ((rng.random(17) * 2 - 1) * 2).astype(np.float32)
    w = (rng.random(17) * 2 - 1).astype(np.float32)
    got = orc.rms_norm(x, w, 1e-5).astype(np.float64)
    inv = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean() + np.float64(np.float32(1e-5)))
    ref = x.astype(np.float64) * inv * w.astype(np.float64)
    assert np.all(np.abs(got - ref) <= (17 + 8) / 2 ** 24 * np.abs(ref))
    s = ((rng.random(64) * 2 - 1) * 8).astype(np.float32)
    ref = s.astype(np.float64) / (1 + np.exp(-s.astype(np.float64)))
    got = orc.silu(s).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 4 / 2 ** 24 * np.abs(ref))
    z = ((rng.random(19) * 2 - 1) * 8).astype(np.float32)
    e = np.exp(z.astype(np.float64) - z.max())
    ref = e / e.sum()
    assert np.all(np.abs(orc.softmax(z) - ref) <= (19 + 8) / 2 ** 24 * np.abs(ref))


def test_block_diagonal_mask_matches_reference_test(orc):
    # src/ncm_mask.zig:48-64
    m = orc.block_diagonal_mask(2, [1, 2], [False, True])
    assert m.shape == (5, 5)
    assert m[0, 0] and not m[0, 1] and not m[0, 2]
    assert m[2, 0] and not m[2, 1] and m[2, 2] and not m[2, 3]
    assert m[3, 3] and m[3, 4] and m[4, 3]


def test_block_causal_mask_adds_coarser_levels(orc):
    diag = orc.block_diagonal_mask(1, [1, 2, 3])
    causal = orc.block_causal_mask(1, [1, 2, 3])
    assert np.all(causal >= diag)
    # the level-2 queries (rows 4..6) see levels 0 and 1 (cols 1..3) but not later ones
    assert causal[4:7, 1:4].all() and not diag[4:7, 1:4].any()
    assert not causal[1, 2:].any()


def test_level_positions_restart(orc):
    # src/ncm_position.zig:154-159
    assert orc.fill_level_positions(2, [1, 2, 3]).tolist() == [0, 1, 0, 0, 1, 0, 1, 2]


def test_rope_positions_reuse_tables(orc):
    # src/ncm_position.zig:120-152: llama3 tables gathered at restarting positions
    inv = orc.rope_llama3(64, 500000.0, 32.0, 1.0, 4.0, 8192)
    c, s = orc.rope_tables(inv, 3)
    pos = [0, 1, 2, 0, 1, 0]
    cg, sg = c[pos], s[pos]
    assert np.array_equal(cg[3], c[0]) and np.array_equal(sg[4], s[1])


def test_rope_default_against_float64(orc):
    # B3-style check (packages/kernels/root.zig:925-945): |err| <= 1e-6 against
    # tables whose angle is the f32 product position * inv_freq (as the
    # transformers golden computes it) and whose cos/sin are exact.
    for hd, theta in [(64, 10000.0), (64, 500000.0), (128, 10000.0)]:
        inv, c, s = orc.rope_default(hd, theta, 4096)
        inv64 = 1.0 / (np.float64(theta) ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
        ang = (np.arange(4096, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float64)
        ref_c = np.concatenate([np.cos(ang)] * 2, axis=1)
        ref_s = np.concatenate([np.sin(ang)] * 2, axis=1)
        assert np.max(np.abs(c - ref_c)) <= 1e-6
        assert np.max(np.abs(s - ref_s)) <= 1e-6
        assert np.max(np.abs(inv - inv64) / inv64) <= 1e-6


def test_attention_fully_masked_query_returns_output_bias(orc):
    # packages/kernels/root.zig:1031-1066
    x = np.array([[2, -3]], np.float32)
    eye = np.array([[1, 0], [0, 1]], np.float32)
    w = {"q_w": eye, "k_w": eye, "v_w": eye, "o_w": eye, "o_b": np.array([0.25, -0.5], np.float32)}
    out = orc.attention(x, w, 1, 1, 2, 1e-5, np.ones((1, 2), np.float32), np.zeros((1, 2), np.float32),
                        np.zeros((1, 1), np.uint8))
    assert np.array_equal(out.ravel(), np.array([0.25, -0.5], np.float32))


def test_tiny_decoder_attention_context(orc):
    # src/decoder.zig:292-364: zero Q/K weights give uniform causal attention,
    # so the context of token 1 is the mean of the two values.
    x = np.array([[0.3, 0.4], [0.7, 0.8]], np.float32)
    zero = np.zeros((2, 2), np.float32)
    eye = np.eye(2, dtype=np.float32)
    w = {"q_w": zero, "k_w": zero, "v_w": eye, "o_w": eye}
    _, c, s = orc.rope_default(2, 10000.0, 2)
    mask = orc.causal_mask(np.arange(2), np.arange(2))
    out = orc.attention(x, w, 1, 1, 2, 1e-5, c, s, mask)
    assert np.allclose(out[0], x[0], atol=1e-6)
    assert np.allclose(out[1], (x[0] + x[1]) / 2, atol=1e-6)


@pytest.mark.parametrize("bf16_mode", [True, False])
def test_attention_rows_equal_full_attention_rows(orc, bf16_mode):
    """The row-subset attention (K/V of every row, Q of the chosen rows) gives
    each chosen row the same bits as orc_attention, which restates
    attention_impl for all rows; block-causal mask, GQA 4:2."""
    rng = np.random.default_rng(21)
    T, hidden, H, Hkv, hd = 96, 128, 4, 2, 64
    x = orc.round_bf16(rng.standard_normal((T, hidden)).astype(np.float32))
    w = {n: orc.round_bf16((rng.standard_normal((o, i)) * 0.05).astype(np.float32))
         for n, o, i in (("q_w", H * hd, hidden), ("k_w", Hkv * hd, hidden), ("v_w", Hkv * hd, hidden),
                         ("o_w", hidden, H * hd))}
    levels = [16, 16, 32, 32]
    pos = np.asarray(orc.fill_level_positions(0, levels), np.int64)
    _, c, s = orc.rope_default(hd, 500000.0, int(pos.max()) + 1)
    mask = orc.block_causal_mask(0, levels).astype(np.uint8)
    full = orc.attention(x, w, H, Hkv, hd, 1e-5, c[pos], s[pos], mask, bf16_mode=bf16_mode)
    rows = [0, 5, 17, 33, 50, 64, 95]
    got = orc.attention_rows(x, w, H, Hkv, hd, c[pos], s[pos], mask, rows, bf16_mode=bf16_mode, threads=3)
    assert np.array_equal(got.view(np.uint32), full[rows].view(np.uint32))


def _golden_npz(name):
    return np.load(GOLDEN / name)


def test_upsample_matches_torch_bit_exact(orc):
    """U_i of the quantiser (vq_forward_semantics.md:82): F.interpolate(size=T),
    linear (align_corners=False) and nearest, against committed torch outputs."""
    z = _golden_npz("upsample.npz")
    cases = [k[2:] for k in z.files if k.startswith("q_")]
    assert len(cases) == 5
    for c in cases:
        B, Tq, D, T = map(int, c.split("_"))
        q = z[f"q_{c}"]
        for mode in ("linear", "nearest"):
            got = orc.upsample(q, T, mode)
            assert np.array_equal(got.view(np.uint32), z[f"{mode}_{c}"].view(np.uint32)), (mode, c)


def test_conv1d_k3_matches_torch(orc):
    """Phi / post-upsample convolution: kernel 3, padding 1, against torch's
    float64 F.conv1d; both the f64-accumulating checker and the restatement of
    apply_post_upsample_conv (src/ncm_model.zig:296-326, f32 in reference order)."""
    z = _golden_npz("conv1d_k3.npz")
    for c in sorted(k[2:] for k in z.files if k.startswith("x_")):
        x, w, b, y = z[f"x_{c}"], z[f"w_{c}"], z[f"b_{c}"], z[f"y_{c}"]
        scale = np.abs(x) @ np.abs(w).sum(axis=2).T + np.abs(b)
        got = orc.conv1d_k3(x, w, b, alpha=0.0, beta=1.0)
        assert np.all(np.abs(got - y) <= 1e-6 * scale + 1e-7), c
        post = orc.apply_post_upsample_conv(x, w, b)
        assert np.all(np.abs(post - (x + y)) <= 1e-5 * (scale + np.abs(x))), c


def test_conv1d_k3_segments_are_independent(orc):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((30, 8)).astype(np.float32)
    w = (rng.standard_normal((8, 8, 3)) * 0.2).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    whole = orc.conv1d_k3(x, w, b, segments=[10, 5, 15], alpha=0.5, beta=0.5)
    parts = [orc.conv1d_k3(x[a:e], w, b, alpha=0.5, beta=0.5) for a, e in ((0, 10), (10, 15), (15, 30))]
    assert np.array_equal(whole, np.concatenate(parts))


def test_scale_update_ex_nearest_without_phi_is_scale_update(orc):
    rng = np.random.default_rng(2)
    B, T, D, K, L, f = 2, 32, 16, 64, 3, 4
    cbs = orc.bf16_bits(rng.standard_normal((L, K, D)).astype(np.float32))
    codes = rng.integers(0, K, size=(L, B * T // f)).astype(np.int32)
    r0 = rng.standard_normal((B * T, D)).astype(np.float32)
    r1, a1 = r0.copy(), np.zeros_like(r0)
    r2, a2 = r0.copy(), np.zeros_like(r0)
    orc.scale_update(codes, cbs, r1, a1, B, T, f)
    orc.scale_update_ex(codes, cbs, r2, a2, B, T, f, mode="nearest")
    assert np.array_equal(r1, r2) and np.array_equal(a1, a2)


def test_group_norm_and_stride4_convs_match_torch(orc):
    """Pre-quant GroupNorm (affine=False) and the level-0 cascade's stride-4
    Conv1d / ConvTranspose1d against committed float64 torch outputs."""
    z = _golden_npz("level0.npz")
    assert np.abs(orc.group_norm(z["gn_x"], 8) - z["gn_y"]).max() < 1e-5
    x, w, b = z["conv_x"], z["conv_w"], z["conv_b"]
    scale = np.abs(x).max() * np.abs(w).sum(axis=(1, 2)).max() + np.abs(b).max()
    assert np.abs(orc.conv_down4(x, w, b) - z["down_y"]).max() <= 1e-6 * scale
    assert np.abs(orc.conv_up4(x, w, b) - z["up_y"]).max() <= 1e-6 * scale


def test_ema_matches_the_spec_equations(orc):
    """One EMA step restated with numpy from vq_forward_semantics.md:141-173."""
    rng = np.random.default_rng(9)
    N, D, K, decay, eps = 500, 16, 40, 0.99, 1e-5
    u = rng.standard_normal((N, D)).astype(np.float32)
    codes = rng.integers(0, K, N).astype(np.int32)
    cnt0 = rng.random(K).astype(np.float32) * 3
    m0 = rng.standard_normal((K, D)).astype(np.float32)
    cnt, m, e, counts, sums = orc.ema(u, codes, cnt0, m0, decay, eps)
    n_k = np.bincount(codes, minlength=K).astype(np.float64)
    s_k = np.zeros((K, D))
    np.add.at(s_k, codes, u.astype(np.float64))
    N_k = decay * cnt0.astype(np.float64) + (1 - decay) * n_k
    n = N_k.sum()
    N_hat = (N_k + eps) / (n + K * eps) * n
    m_k = decay * m0.astype(np.float64) + (1 - decay) * s_k
    assert np.array_equal(counts, n_k.astype(np.float32))
    assert np.allclose(sums, s_k, atol=1e-4)
    assert np.allclose(cnt, N_k, rtol=1e-6)
    assert np.allclose(e, m_k / N_hat[:, None], rtol=1e-5, atol=1e-6)
