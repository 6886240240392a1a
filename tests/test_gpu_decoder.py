"""GPU parity of the NCM decoder pieces (L3-L6, config 4) against the oracle.

The attention check runs the oracle's restatement of attention_impl in bf16
mode (packages/kernels/root.zig:450-581) with 0/1 selection matrices as the
Q/K/V/O projections, so the oracle sees exactly the GPU's Q, K and V and the
comparison isolates RoPE, masking, softmax and the P.V product. The GPU uses
an online softmax whose bf16 probabilities are unnormalised, so contexts are
held to a bf16 bar, not bit equality:
    |gpu - oracle| <= 2e-2 |oracle| + 1e-2 max|V|
"""
import numpy as np
import pytest
import torch

from helpers import check_gemm, from_dev_bf16, gen_bf16, to_dev_bf16

pytestmark = pytest.mark.gpu


def _selection(rows_from: int, width: int, count: int) -> np.ndarray:
    w = np.zeros((count, width), np.float32)
    w[np.arange(count), rows_from + np.arange(count)] = 1.0
    return w


def oracle_attention_core(orc, qkv_bits, H, Hkv, cos, sin, mask_bool, q_norm=None, k_norm=None, eps=1e-5):
    """Context [T, H*64] from qkv rows via orc_attention with selection
    projections (and QK-norm scales, when given)."""
    T, width = qkv_bits.shape
    x = orc.bf16_widen(qkv_bits)
    w = {
        "q_w": _selection(0, width, H * 64),
        "k_w": _selection(H * 64, width, Hkv * 64),
        "v_w": _selection((H + Hkv) * 64, width, Hkv * 64),
        # output projection: identity onto the first H*64 columns of a width-wide output
        "o_w": _selection(0, H * 64, H * 64) if width == H * 64 else np.vstack(
            [np.eye(H * 64, dtype=np.float32), np.zeros((width - H * 64, H * 64), np.float32)]),
    }
    if q_norm is not None:
        w["q_norm"], w["k_norm"] = q_norm, k_norm
    out = orc.attention(x, w, H, Hkv, 64, eps, cos, sin, mask_bool.astype(np.uint8), bf16_mode=True)
    return out[:, : H * 64]


def _mask_case(orc, mode, T, prefix=0, levels=(), pad=(), window=None):
    from ncmorph_b200.ncm_model import level_positions, make_mask
    if mode == "causal":
        mb = orc.causal_mask(np.arange(T), np.arange(T), window or 0)
        pos = np.arange(T, dtype=np.int32)
        return make_mask(mode, prefix, levels, pad, sliding_window=window), mb, pos
    elif mode == "block_diagonal":
        mb = orc.block_diagonal_mask(prefix, list(levels), list(pad))
        pos = level_positions(prefix, levels)
    else:
        mb = orc.block_causal_mask(prefix, list(levels), list(pad))
        pos = level_positions(prefix, levels)
    return make_mask(mode, prefix, levels, pad), mb, pos


@pytest.mark.parametrize("mode,T,prefix,levels,pad,H,Hkv", [
    ("causal", 256, 0, (), (), 4, 2),
    ("block_diagonal", 256, 2, (14, 16, 32, 64, 128), (False, True), 4, 2),
    ("block_causal", 256, 0, (16, 16, 32, 64, 128), (), 8, 2),
    ("block_causal", 200, 1, (7, 32, 160), (False,), 4, 1),
    ("causal", 384, 0, (), (), 2, 2),
])
def test_attention_matches_oracle(orc, cuda_dev, mode, T, prefix, levels, pad, H, Hkv):
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(T + H)
    width = (H + 2 * Hkv) * 64
    qkv_bits = gen_bf16(rng, (T, width))
    mask, mb, pos = _mask_case(orc, mode, T, prefix, levels, pad)
    cos, sin = ncm_model.rope_tables(64, 500000.0, pos)
    qkv = to_dev_bf16(qkv_bits, cuda_dev)
    ctx = ncm_model.attention_bf16(qkv, H, Hkv, mask, torch.from_numpy(cos).to(cuda_dev),
                                   torch.from_numpy(sin).to(cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(ctx))
    ref = oracle_attention_core(orc, qkv_bits, H, Hkv, cos, sin, mb)
    # RoPE was applied in place: Q/K columns must equal the oracle's rotate_head (bf16 mode) bit for bit
    vmax = np.abs(orc.bf16_widen(qkv_bits[:, (H + Hkv) * 64:])).max()
    err = np.abs(got - ref)
    tol = 2e-2 * np.abs(ref) + 1e-2 * vmax
    bad = np.argwhere(err > tol)
    assert bad.size == 0, f"{len(bad)} context elements outside the bar; first {bad[0]} got {got[tuple(bad[0])]} ref {ref[tuple(bad[0])]}"
    print(f"{mode} T={T}: max |err| {err.max():.3g}, mean {err.mean():.3g}")


@pytest.mark.parametrize("T,window,H,Hkv", [(384, 100, 4, 2), (512, 128, 2, 1), (1024, 300, 4, 1),
                                             (264, 1, 2, 2), (256, 4096, 2, 1)])
def test_attention_sliding_window_matches_oracle(orc, cuda_dev, T, window, H, Hkv):
    """Causal attention with a sliding window (causal_mask, root.zig:380-399:
    q - W < k <= q): windows inside a tile, on a tile boundary, across
    several tiles, of one key, and wider than the sequence; key tiles left of
    every query's window are skipped."""
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(T + window)
    width = (H + 2 * Hkv) * 64
    qkv_bits = gen_bf16(rng, (T, width))
    mask, mb, pos = _mask_case(orc, "causal", T, window=window)
    cos, sin = ncm_model.rope_tables(64, 10000.0, pos)
    ctx = ncm_model.attention_bf16(to_dev_bf16(qkv_bits, cuda_dev), H, Hkv, mask, torch.from_numpy(cos).to(cuda_dev),
                                   torch.from_numpy(sin).to(cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(ctx))
    ref = oracle_attention_core(orc, qkv_bits, H, Hkv, cos, sin, mb)
    vmax = np.abs(orc.bf16_widen(qkv_bits[:, (H + Hkv) * 64:])).max()
    err = np.abs(got - ref)
    bad = np.argwhere(err > 2e-2 * np.abs(ref) + 1e-2 * vmax)
    assert bad.size == 0, f"{len(bad)} context elements outside the bar; first {bad[0]}"
    if window == 1:
        # one key: the context is that row's own V head, rounded
        v = orc.bf16_widen(qkv_bits[:, (H + Hkv) * 64:])
        for hh in range(H):
            kv = hh // (H // Hkv)
            assert np.array_equal(got[:, hh * 64:(hh + 1) * 64], v[:, kv * 64:(kv + 1) * 64])


def test_sliding_window_only_in_causal_mode(cuda_dev):
    from ncmorph_b200 import _lib, ncm_model
    qkv = torch.zeros((64, 256), dtype=torch.bfloat16, device=cuda_dev)
    for mask in (ncm_model.make_mask("block_causal", 0, (32, 32), sliding_window=8),
                 ncm_model.make_mask("causal", sliding_window=-1)):
        with pytest.raises(_lib.NcmError) as e:
            ncm_model.attention_bf16(qkv, 2, 1, mask)
        assert e.value.status == _lib.NCM_EINVAL


@pytest.mark.parametrize("step", [128, 512])
def test_attention_running_maximum_jumps(orc, cuda_dev, step):
    """Scores that rise tile by tile, so the running reference maximum lags
    (step 128: by 23 per tile in the log2 domain, moved every third tile)
    or moves at every tile (step 512: 92 per tile, O rescaled by 2^-92).
    Integer-valued Q and K without RoPE make every score exact in f32 and in
    bf16, so the GPU and the oracle round the same scores."""
    from ncmorph_b200 import _lib, ncm_model
    T, H, Hkv = 512, 2, 1
    rng = np.random.default_rng(step)
    x = np.zeros((T, (H + 2 * Hkv) * 64), np.float32)
    x[:, 0:8] = 1.0                      # query head 0: ones on the first 8 dims
    x[:, 64:72] = 1.0                    # query head 1
    t = np.arange(T)
    x[:, H * 64:H * 64 + 8] = (step // 8 * (t // 128) + t % 8)[:, None]   # key: q.k = step * tile + 8 (t % 8)
    x[:, (H + Hkv) * 64:] = rng.standard_normal((T, Hkv * 64))
    qkv_bits = orc.bf16_bits(x)
    assert np.array_equal(orc.bf16_widen(qkv_bits)[:, H * 64:H * 64 + 8], x[:, H * 64:H * 64 + 8])
    mask = ncm_model.make_mask("causal", 0, (), ())
    ctx = ncm_model.attention_bf16(to_dev_bf16(qkv_bits, cuda_dev), H, Hkv, mask)
    got = orc.bf16_widen(from_dev_bf16(ctx))
    cos = np.ones((T, 64), np.float32)
    sin = np.zeros((T, 64), np.float32)
    ref = oracle_attention_core(orc, qkv_bits, H, Hkv, cos, sin, orc.causal_mask(t, t))
    err = np.abs(got - ref)
    assert np.all(err <= 2e-2 * np.abs(ref) + 1e-2 * np.abs(x[:, (H + Hkv) * 64:]).max()), err.max()


def test_rope_in_place_matches_rotate_head(orc, cuda_dev):
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(3)
    T, H, Hkv = 64, 2, 1
    width = (H + 2 * Hkv) * 64
    qkv_bits = gen_bf16(rng, (T, width))
    pos = ncm_model.level_positions(0, (32, 32))
    cos, sin = ncm_model.rope_tables(64, 10000.0, pos)
    qkv = to_dev_bf16(qkv_bits, cuda_dev)
    mask = ncm_model.make_mask("block_diagonal", 0, (32, 32))
    ncm_model.attention_bf16(qkv, H, Hkv, mask, torch.from_numpy(cos).to(cuda_dev), torch.from_numpy(sin).to(cuda_dev))
    got = from_dev_bf16(qkv)
    # oracle rotate_head via attention's Q path: project Q with identity, read it back through a 1-key mask? simpler:
    # restate rotate_head (root.zig:615-633) here in f32 with bf16 rounding at each step
    def rb(a):
        return orc.round_bf16(np.asarray(a, np.float32))
    x = orc.bf16_widen(qkv_bits).copy()
    for hh in range(H + Hkv):
        v = x[:, hh * 64:(hh + 1) * 64]
        first, second = v[:, :32].copy(), v[:, 32:].copy()
        cf, sf, cs, ss = rb(cos[:, :32]), rb(sin[:, :32]), rb(cos[:, 32:]), rb(sin[:, 32:])
        left, right = rb(first * cf), rb(-second * sf)
        right2, left2 = rb(first * ss), rb(second * cs)
        v[:, :32] = rb(left + right)
        v[:, 32:] = rb(left2 + right2)
    assert np.array_equal(got[:, : (H + Hkv) * 64], orc.bf16_bits(x[:, : (H + Hkv) * 64]))
    assert np.array_equal(got[:, (H + Hkv) * 64:], qkv_bits[:, (H + Hkv) * 64:])  # V untouched


def _oracle_qk_norm_rope(orc, qkv_bits, H, Hkv, qn, kn, eps, cos, sin):
    """Q and K columns after attention_impl's per-head rms_norm_bf16 and
    rotate_head (root.zig:500-530), from the oracle's own functions."""
    x = orc.bf16_widen(qkv_bits)[:, : (H + Hkv) * 64].copy()
    T = x.shape[0]
    for t in range(T):
        for hh in range(H + Hkv):
            x[t, hh * 64:(hh + 1) * 64] = orc.rms_norm(x[t, hh * 64:(hh + 1) * 64], qn if hh < H else kn, eps,
                                                       bf16_mode=True)
    x = np.ascontiguousarray(x)
    if cos is not None:
        orc.lib().orc_rotate_rows(x, T, H + Hkv, 64, np.ascontiguousarray(cos, np.float32),
                                  np.ascontiguousarray(sin, np.float32), 1)
    return orc.bf16_bits(x)


@pytest.mark.parametrize("T,H,Hkv,rope,scale", [(256, 4, 2, True, 1.0), (200, 2, 1, False, 1.0),
                                                (64, 8, 2, True, 1e-3), (64, 2, 2, True, 40.0)])
def test_qk_norm_then_rope_bit_exact(orc, cuda_dev, T, H, Hkv, rope, scale):
    """Per-head RMSNorm with q_norm / k_norm, then RoPE, in place: every Q and
    K element equals the oracle's rms_norm_bf16 + rotate_head bit for bit (the
    GPU keeps the reference's sum-of-squares order), V stays untouched. The
    scale moves the heads' magnitude (tiny and large rows)."""
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(T * 7 + H)
    width = (H + 2 * Hkv) * 64
    qkv_bits = orc.bf16_bits(orc.bf16_widen(gen_bf16(rng, (T, width))) * np.float32(scale))
    qn = gen_bf16(rng, (64,))
    kn = gen_bf16(rng, (64,))
    eps = 1e-6
    pos = ncm_model.level_positions(0, (T // 2, T - T // 2))
    cos, sin = ncm_model.rope_tables(64, 1000000.0, pos) if rope else (None, None)
    qkv = to_dev_bf16(qkv_bits, cuda_dev)
    mask = ncm_model.make_mask("block_causal", 0, (T // 2, T - T // 2))
    dev = (lambda a: None if a is None else torch.from_numpy(a).to(cuda_dev))  # noqa: E731
    ncm_model.attention_bf16(qkv, H, Hkv, mask, dev(cos), dev(sin), q_norm=to_dev_bf16(qn, cuda_dev),
                             k_norm=to_dev_bf16(kn, cuda_dev), eps=eps)
    got = from_dev_bf16(qkv)
    ref = _oracle_qk_norm_rope(orc, qkv_bits, H, Hkv, orc.bf16_widen(qn), orc.bf16_widen(kn), eps, cos, sin)
    diff = np.argwhere(got[:, : (H + Hkv) * 64] != ref)
    assert diff.size == 0, f"{len(diff)} Q/K elements differ; first {diff[0]}"
    assert np.array_equal(got[:, (H + Hkv) * 64:], qkv_bits[:, (H + Hkv) * 64:])


@pytest.mark.parametrize("mode,T,prefix,levels,pad,H,Hkv", [
    ("block_causal", 256, 0, (16, 16, 32, 64, 128), (), 4, 2),
    ("block_diagonal", 200, 1, (7, 32, 160), (True,), 2, 1),
])
def test_attention_qk_norm_matches_oracle(orc, cuda_dev, mode, T, prefix, levels, pad, H, Hkv):
    """ncm_attention_qk_norm_bf16 against attention_impl with
    query_norm_weight / key_norm_weight (root.zig:450-581, bf16 mode)."""
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(T + 11 * H)
    width = (H + 2 * Hkv) * 64
    qkv_bits = gen_bf16(rng, (T, width))
    qn = orc.bf16_bits(1.0 + 0.2 * rng.standard_normal(64).astype(np.float32))
    kn = orc.bf16_bits(1.0 + 0.2 * rng.standard_normal(64).astype(np.float32))
    eps = 1e-6
    mask, mb, pos = _mask_case(orc, mode, T, prefix, levels, pad)
    cos, sin = ncm_model.rope_tables(64, 1000000.0, pos)
    qkv = to_dev_bf16(qkv_bits, cuda_dev)
    ctx = ncm_model.attention_bf16(qkv, H, Hkv, mask, torch.from_numpy(cos).to(cuda_dev),
                                   torch.from_numpy(sin).to(cuda_dev), q_norm=to_dev_bf16(qn, cuda_dev),
                                   k_norm=to_dev_bf16(kn, cuda_dev), eps=eps)
    got = orc.bf16_widen(from_dev_bf16(ctx))
    ref = oracle_attention_core(orc, qkv_bits, H, Hkv, cos, sin, mb, orc.bf16_widen(qn), orc.bf16_widen(kn), eps)
    vmax = np.abs(orc.bf16_widen(qkv_bits[:, (H + Hkv) * 64:])).max()
    err = np.abs(got - ref)
    bad = np.argwhere(err > 2e-2 * np.abs(ref) + 1e-2 * vmax)
    assert bad.size == 0, f"{len(bad)} context elements outside the bar; first {bad[0]}"


def test_attention_qk_norm_needs_both_scales(cuda_dev):
    from ncmorph_b200 import _lib, ncm_model
    qkv = torch.zeros((64, 256), dtype=torch.bfloat16, device=cuda_dev)
    qn = torch.ones((64,), dtype=torch.bfloat16, device=cuda_dev)
    mask = ncm_model.make_mask("causal", 0, (), ())
    with pytest.raises(_lib.NcmError) as e:
        ncm_model.attention_bf16(qkv, 2, 1, mask, q_norm=qn)
    assert e.value.status == _lib.NCM_EINVAL


def test_rope_tables_bit_exact(orc):
    from ncmorph_b200 import ncm_model
    pos = ncm_model.level_positions(1, (3, 5))
    c, s = ncm_model.rope_tables(64, 500000.0, pos)
    _, oc, os_ = orc.rope_default(64, 500000.0, int(pos.max()) + 1)
    assert np.array_equal(c, oc[pos]) and np.array_equal(s, os_[pos])


def test_rms_norm_within_one_ulp(orc, cuda_dev):
    from ncmorph_b200 import ncm_model
    rng = np.random.default_rng(8)
    rows, width = 300, 2048
    x = gen_bf16(rng, (rows, width), 3.0)
    w = gen_bf16(rng, (width,))
    y = from_dev_bf16(ncm_model.rms_norm_bf16(to_dev_bf16(x, cuda_dev), to_dev_bf16(w, cuda_dev), 1e-5))
    ref = np.stack([orc.bf16_bits(orc.rms_norm(orc.bf16_widen(x[r]), orc.bf16_widen(w), 1e-5, bf16_mode=True))
                    for r in range(rows)])
    diff = np.abs(y.astype(np.int32) - ref.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.99


def test_embedding_gather_and_range(cuda_dev):
    from ncmorph_b200 import _lib, device, ncm_model
    table = torch.randn((50, 16), device=cuda_dev).to(torch.bfloat16)
    ids = torch.tensor([3, 0, 49, 7], dtype=torch.int32, device=cuda_dev)
    out = ncm_model.embedding_gather(table, ids)
    assert torch.equal(out.view(torch.int16), table[ids.long()].view(torch.int16))
    ncm_model.embedding_gather(table, torch.tensor([50], dtype=torch.int32, device=cuda_dev))
    with pytest.raises(_lib.NcmError) as ei:
        device.sync(cuda_dev)
    assert ei.value.status == _lib.NCM_ERANGE


# --------------------------------------------------------- full forward
def _rand_weights(cfg, dev, seed, layers):
    from ncmorph_b200.ncm_model import LayerWeights, Weights
    g = torch.Generator(device=dev).manual_seed(seed)

    def r(*shape, s=0.02):
        return (torch.randn(shape, generator=g, device=dev) * s).to(torch.bfloat16)

    def ones(n):
        return (1.0 + 0.1 * torch.randn((n,), generator=g, device=dev)).to(torch.bfloat16)

    Hd, V, F = cfg.hidden_size, cfg.vq_width, cfg.intermediate_size
    qkvw = (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * 64
    Ls = [LayerWeights(ln_1=ones(Hd), qkv=r(qkvw, Hd), o=r(Hd, cfg.num_attention_heads * 64), ln_2=ones(Hd),
                       gate_up=r(2 * F, Hd), down=r(Hd, F)) for _ in range(layers)]
    return Weights(input_projection=r(Hd, V), input_projection_bias=r(Hd, s=0.1),
                   level_embedding=r(len(cfg.level_lengths), Hd, s=0.1), final_norm=ones(Hd), layers=Ls)


def _oracle_rope(orc, cfg):
    """cos/sin rows at the per-level restarting positions: rope_default, or
    rope_llama3's frequencies when the config carries Llama 3 scaling."""
    pos = np.asarray(orc.fill_level_positions(cfg.prefix_length, list(cfg.level_lengths)), np.int64)
    if cfg.rope_llama3 is None:
        _, ct, st = orc.rope_default(64, cfg.rope_theta, int(pos.max()) + 1)
    else:
        ct, st = orc.rope_tables(orc.rope_llama3(64, cfg.rope_theta, *cfg.rope_llama3), int(pos.max()) + 1)
    return ct[pos], st[pos]


def oracle_ncm_forward(orc, cfg, w, inputs_bits):
    """ncm_model.forward (src/ncm_model.zig:89-250) with the bf16 layer of decoder.zig:168-216."""
    f = lambda t: orc.bf16_widen(from_dev_bf16(t))  # noqa: E731
    rb = orc.round_bf16
    T = cfg.seq_len
    x = orc.bf16_widen(inputs_bits).astype(np.float32)
    if w.post_conv_weight is not None:
        # ncm_model.zig:141-153: each level's rows get apply_post_upsample_conv with its own kernel
        pw = f(w.post_conv_weight)
        pb = w.post_conv_bias.cpu().numpy()
        off = cfg.prefix_length
        for i, n in enumerate(cfg.level_lengths):
            x[off:off + n] = orc.apply_post_upsample_conv(x[off:off + n], pw[i], pb[i])
            off += n
    h = orc.matmul_bf16(x, f(w.input_projection), f(w.input_projection_bias), threads=8)
    emb = f(w.level_embedding)
    off = cfg.prefix_length
    for i, n in enumerate(cfg.level_lengths):
        if cfg.use_level_encoding:
            h[off:off + n] = rb(h[off:off + n] + emb[i])
        off += n
    cos, sin = _oracle_rope(orc, cfg)
    if cfg.mask == "causal":
        # source_causal (ncm_model.zig:199-203): sequence order, optional window
        mask = orc.causal_mask(np.arange(T), np.arange(T), cfg.sliding_window or 0)
    else:
        mask = (orc.block_causal_mask if cfg.mask == "block_causal" else orc.block_diagonal_mask)(
            cfg.prefix_length, list(cfg.level_lengths))
    H, Hkv, F = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    eps = cfg.rms_norm_epsilon

    def norm_rows(x, wt):
        return np.stack([orc.rms_norm(x[i], wt, eps, bf16_mode=True) for i in range(x.shape[0])])

    for L in w.layers:
        n = norm_rows(h, f(L.ln_1))
        qkv = f(L.qkv)
        aw = {"q_w": qkv[: H * 64], "k_w": qkv[H * 64:(H + Hkv) * 64], "v_w": qkv[(H + Hkv) * 64:], "o_w": f(L.o)}
        if L.q_norm is not None:
            aw["q_norm"], aw["k_norm"] = f(L.q_norm), f(L.k_norm)
        att = orc.attention(n, aw, H, Hkv, 64, eps, cos, sin, mask.astype(np.uint8), bf16_mode=True)
        h = rb(h + att)
        n = norm_rows(h, f(L.ln_2))
        gu = f(L.gate_up)
        g = orc.matmul_bf16(n, gu[:F], threads=8)
        u = orc.matmul_bf16(n, gu[F:], threads=8)
        act = rb(orc.silu_bf16(g) * u)
        h = rb(h + orc.matmul_bf16(act, f(L.down), threads=8))
    return norm_rows(h, f(w.final_norm))


@pytest.mark.parametrize("mask,prefix,levels", [("block_causal", 0, (16, 16, 32, 64, 128)),
                                                ("block_diagonal", 0, (32, 32, 64, 128))])
def test_ncm_forward_small_matches_oracle(orc, cuda_dev, mask, prefix, levels):
    from ncmorph_b200 import ncm_model
    cfg = ncm_model.Config(hidden_size=256, vq_width=64, num_attention_heads=4, num_key_value_heads=2,
                           intermediate_size=512, level_lengths=levels, prefix_length=prefix, mask=mask)
    w = _rand_weights(cfg, cuda_dev, 5, layers=2)
    rng = np.random.default_rng(6)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    out = ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(out))
    ref = oracle_ncm_forward(orc, cfg, w, inputs)
    _assert_rows_within(got, ref, f"ncm forward {mask}")


@pytest.mark.parametrize("prefix,levels,window", [(2, (16, 16, 32, 64, 126), None), (0, (16, 16, 32, 64, 128), 96),
                                                  (1, (7, 32), 8)])
def test_ncm_forward_source_causal_matches_oracle(orc, cuda_dev, prefix, levels, window):
    """ncm_model with source_causal (src/ncm_model.zig:199-203): causal in
    sequence order with an optional sliding window, while RoPE positions and
    level embeddings still follow the levels."""
    from ncmorph_b200 import ncm_model
    cfg = ncm_model.Config(hidden_size=256, vq_width=64, num_attention_heads=4, num_key_value_heads=2,
                           intermediate_size=512, level_lengths=levels, prefix_length=prefix, mask="causal",
                           sliding_window=window)
    w = _rand_weights(cfg, cuda_dev, 11, layers=2)
    rng = np.random.default_rng(12)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    out = ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(out))
    ref = oracle_ncm_forward(orc, cfg, w, inputs)
    _assert_rows_within(got, ref, f"ncm forward source_causal window {window}")


@pytest.mark.parametrize("levels", [(16, 16, 32, 64, 128), (8, 8, 16)])
def test_ncm_forward_qk_norm_matches_oracle(orc, cuda_dev, levels):
    """Layers with q_norm / k_norm (ncm_model.zig:42-43, as Qwen3-style
    checkpoints carry): the projection runs without the RoPE epilogue and the
    per-head norm + RoPE kernel follows it; 256 rows and 32 rows (the swapped
    GEMM form)."""
    from ncmorph_b200 import ncm_model
    cfg = ncm_model.Config(hidden_size=256, vq_width=64, num_attention_heads=4, num_key_value_heads=2,
                           intermediate_size=512, level_lengths=levels, prefix_length=0, mask="block_causal")
    w = _rand_weights(cfg, cuda_dev, 8, layers=2)
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    for L in w.layers:
        L.q_norm = (1.0 + 0.2 * torch.randn((64,), generator=g, device=cuda_dev)).to(torch.bfloat16)
        L.k_norm = (1.0 + 0.2 * torch.randn((64,), generator=g, device=cuda_dev)).to(torch.bfloat16)
    rng = np.random.default_rng(10)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    out = ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(out))
    ref = oracle_ncm_forward(orc, cfg, w, inputs)
    _assert_rows_within(got, ref, "ncm forward with QK-norm")


def test_ncm_forward_decode_size_split_k_matches_oracle(orc, cuda_dev):
    """40 positions (at most 64 rows: the swapped GEMM form) and a width that
    makes the projections split K, so the f32 partial reduction carries the
    bias, the residual adds and the output rounding."""
    from ncmorph_b200 import ncm_model
    cfg = ncm_model.Config(hidden_size=1024, vq_width=64, num_attention_heads=16, num_key_value_heads=4,
                           intermediate_size=2048, level_lengths=(8, 16, 16), prefix_length=0, mask="block_causal")
    w = _rand_weights(cfg, cuda_dev, 7, layers=2)
    rng = np.random.default_rng(8)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    out = ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(out))
    ref = oracle_ncm_forward(orc, cfg, w, inputs)
    _assert_rows_within(got, ref, "ncm forward, decode size")


def test_ncm_forward_post_upsample_convs_match_oracle(orc, cuda_dev):
    """weights.post_upsample_convs (ncm_model.zig:141-153): each level's input
    rows pass through x + bias + Conv1d_k3(x) with that level's kernel first."""
    from ncmorph_b200 import ncm_model
    levels = (16, 16, 32, 64, 128)
    cfg = ncm_model.Config(hidden_size=256, vq_width=64, num_attention_heads=4, num_key_value_heads=2,
                           intermediate_size=512, level_lengths=levels, prefix_length=0, mask="block_causal")
    w = _rand_weights(cfg, cuda_dev, 7, layers=2)
    g = torch.Generator(device=cuda_dev).manual_seed(8)
    w.post_conv_weight = (torch.randn((len(levels), 64, 64, 3), generator=g, device=cuda_dev) * 0.05).to(
        torch.bfloat16)
    w.post_conv_bias = torch.randn((len(levels), 64), generator=g, device=cuda_dev) * 0.1
    rng = np.random.default_rng(9)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    out = ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))
    got = orc.bf16_widen(from_dev_bf16(out))
    ref = oracle_ncm_forward(orc, cfg, w, inputs)
    _assert_rows_within(got, ref, "ncm forward, post-upsample convs")
    # the convolutions change the result (they are not skipped)
    w.post_conv_weight.zero_()
    w.post_conv_bias.zero_()
    plain = orc.bf16_widen(from_dev_bf16(ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))))
    assert np.abs(plain - got).max() > 0.1


def test_ncm_forward_llama3_rope_matches_oracle(orc, cuda_dev):
    """The forward with Llama 3 scaled RoPE frequencies (rope_llama3,
    root.zig:636-666; Llama-3.2-1B's scaling) against the oracle built from
    the same frequencies; the scaling must change the result."""
    from ncmorph_b200 import ncm_model
    levels = (16, 16, 32, 64, 128)
    base = dict(hidden_size=256, vq_width=64, num_attention_heads=4, num_key_value_heads=2, intermediate_size=512,
                level_lengths=levels, prefix_length=0, mask="block_causal", rope_theta=10000.0)
    cfg = ncm_model.Config(**base, rope_llama3=(8.0, 1.0, 4.0, 64))
    w = _rand_weights(cfg, cuda_dev, 13, layers=2)
    rng = np.random.default_rng(14)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    got = orc.bf16_widen(from_dev_bf16(ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))))
    ref = oracle_ncm_forward(orc, cfg, w, inputs)
    _assert_rows_within(got, ref, "llama3 rope")
    plain = orc.bf16_widen(from_dev_bf16(ncm_model.forward(ncm_model.Config(**base), w,
                                                           to_dev_bf16(inputs, cuda_dev))))
    assert np.abs(plain - got).max() > 0


def _assert_rows_within(got, ref, what, rel=2e-2, elem_rms=5e-2):
    """north_star's 2e-2 relative bar per output row (L2 norm of the error
    over the row's norm). Single elements of a layer's bf16 chain (bf16
    scores, probabilities, context, activations, each rounded after sums in
    a different order than the reference's) drift by a few bf16 ulps of the
    row's scale, so elementwise the bar is 2e-2 of |ref| plus 5e-2 of the
    row's RMS: a gross error in any element still fails."""
    err = np.abs(got - ref)
    row_rel = np.sqrt((err ** 2).sum(axis=1)) / np.maximum(np.sqrt((ref ** 2).sum(axis=1)), 1e-30)
    rms = np.sqrt((ref ** 2).mean(axis=1, keepdims=True))
    elem_bad = (err > rel * np.abs(ref) + elem_rms * rms).mean()
    print(f"{what}: worst row relative error {row_rel.max():.3e}, elements outside the bar {elem_bad:.2e}, "
          f"max |err| {err.max():.3g}")
    assert row_rel.max() <= rel
    assert elem_bad == 0.0


def test_config4_layer0_full_size_matches_oracle(orc, cuda_dev):
    """BASELINE config 4 at full size (T = 4096, d = 2048, 32/8 heads, FFN 8192,
    block-causal over levels 256/256/512/1024/2048) with one layer: 80 query
    rows sampled across all five levels against the oracle's composition of
    src/ncm_model.zig:89-250 (K and V of every row, the sampled rows' queries,
    attention_impl root.zig:537-575, O projection, SwiGLU FFN, final norm)."""
    import os
    from ncmorph_b200 import ncm_model
    cfg = ncm_model.Config(hidden_size=2048, vq_width=1024, num_attention_heads=32, num_key_value_heads=8,
                           intermediate_size=8192, level_lengths=(256, 256, 512, 1024, 2048), mask="block_causal")
    w = _rand_weights(cfg, cuda_dev, 17, layers=1)
    rng = np.random.default_rng(18)
    inputs = gen_bf16(rng, (cfg.seq_len, cfg.vq_width))
    got_all = orc.bf16_widen(from_dev_bf16(ncm_model.forward(cfg, w, to_dev_bf16(inputs, cuda_dev))))
    starts = np.cumsum((0,) + cfg.level_lengths)
    rows = []
    for i, n in enumerate(cfg.level_lengths):   # first, last and 14 random rows of every level
        rows += [starts[i], starts[i] + n - 1] + sorted(rng.choice(np.arange(starts[i] + 1, starts[i] + n - 1), 14,
                                                                   replace=False).tolist())
    rows = np.asarray(rows, np.int64)
    threads = max(1, min(32, os.cpu_count() or 1))
    f = lambda t: orc.bf16_widen(from_dev_bf16(t))  # noqa: E731
    rb = orc.round_bf16
    H, Hkv, F, eps = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.rms_norm_epsilon
    x = orc.bf16_widen(inputs).astype(np.float32)
    h = orc.matmul_bf16(x, f(w.input_projection), f(w.input_projection_bias), threads=threads)
    emb = f(w.level_embedding)
    for i, n in enumerate(cfg.level_lengths):
        h[starts[i]:starts[i] + n] = rb(h[starts[i]:starts[i] + n] + emb[i])
    L = w.layers[0]
    n_all = np.stack([orc.rms_norm(h[i], f(L.ln_1), eps, bf16_mode=True) for i in range(h.shape[0])])
    qkv = f(L.qkv)
    aw = {"q_w": qkv[: H * 64], "k_w": qkv[H * 64:(H + Hkv) * 64], "v_w": qkv[(H + Hkv) * 64:], "o_w": f(L.o)}
    cos, sin = _oracle_rope(orc, cfg)
    mask = orc.block_causal_mask(0, list(cfg.level_lengths)).astype(np.uint8)
    att = orc.attention_rows(n_all, aw, H, Hkv, 64, cos, sin, mask, rows, bf16_mode=True, threads=threads)
    hs = rb(h[rows] + att)
    n2 = np.stack([orc.rms_norm(hs[i], f(L.ln_2), eps, bf16_mode=True) for i in range(hs.shape[0])])
    gu = f(L.gate_up)
    g = orc.matmul_bf16(n2, gu[:F], threads=threads)
    u = orc.matmul_bf16(n2, gu[F:], threads=threads)
    act = rb(orc.silu_bf16(g) * u)
    hs = rb(hs + orc.matmul_bf16(act, f(L.down), threads=threads))
    ref = np.stack([orc.rms_norm(hs[i], f(w.final_norm), eps, bf16_mode=True) for i in range(hs.shape[0])])
    _assert_rows_within(got_all[rows], ref, "config 4 layer 0")


def test_config4_forward_runs_and_is_normalised(cuda_dev):
    """BASELINE config 4 shapes: 16 layers, d=2048, 32/8 heads, FFN 8192, 4096 positions, block-causal."""
    from ncmorph_b200 import device, ncm_model
    cfg = ncm_model.Config(hidden_size=2048, vq_width=1024, num_attention_heads=32, num_key_value_heads=8,
                           intermediate_size=8192, level_lengths=(256, 256, 512, 1024, 2048), mask="block_causal")
    w = _rand_weights(cfg, cuda_dev, 9, layers=16)
    for L in w.layers:
        L.ln_1.fill_(1.0)
        L.ln_2.fill_(1.0)
    w.final_norm.fill_(1.0)
    codes = torch.randint(0, 4096, (cfg.seq_len,), dtype=torch.int32, device=cuda_dev)
    table = (torch.randn((4096, cfg.vq_width), device=cuda_dev)).to(torch.bfloat16)
    inputs = ncm_model.embedding_gather(table, codes)
    out = ncm_model.forward(cfg, w, inputs)
    device.sync(cuda_dev)
    o = out.float()
    assert torch.isfinite(o).all()
    rms = o.pow(2).mean(dim=1).sqrt()
    assert torch.allclose(rms, torch.ones_like(rms), atol=2e-2)


def test_qkv_projection_rope_equals_linear_then_rope(orc, cuda_dev):
    """The fused QKV epilogue (RoPE + V transpose) is bit-identical to the
    separate projection and the RoPE that ncm_attention_bf16 applies."""
    import ctypes
    from ncmorph_b200 import _lib, device, kernels, ncm_model
    T, hidden, H, Hkv = 320, 256, 4, 2
    g = torch.Generator(device=cuda_dev).manual_seed(12)
    x = torch.randn((T, hidden), generator=g, device=cuda_dev).to(torch.bfloat16)
    w = (torch.randn(((H + 2 * Hkv) * 64, hidden), generator=g, device=cuda_dev) * 0.05).to(torch.bfloat16)
    pos = ncm_model.level_positions(0, (64, 64, 64, 128))
    c, s = ncm_model.rope_tables(64, 500000.0, pos)
    cd, sd = torch.from_numpy(c).to(cuda_dev), torch.from_numpy(s).to(cuda_dev)
    qkv = torch.empty((T, (H + 2 * Hkv) * 64), dtype=torch.bfloat16, device=cuda_dev)
    vt = torch.empty((Hkv * 64, T), dtype=torch.bfloat16, device=cuda_dev)
    _lib.call("ncm_qkv_projection_rope", device.context(cuda_dev), x.data_ptr(), w.data_ptr(), None, cd.data_ptr(),
              sd.data_ptr(), qkv.data_ptr(), vt.data_ptr(), T, hidden, H, Hkv, device.stream_of(x))
    ref = kernels.linear_bf16(x, w)
    mask = ncm_model.make_mask("causal")
    ncm_model.attention_bf16(ref, H, Hkv, mask, cos=cd, sin=sd)   # applies RoPE to ref in place
    torch.cuda.synchronize()
    assert torch.equal(qkv.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(vt.view(torch.int16), ref[:, (H + Hkv) * 64:].t().contiguous().view(torch.int16))
