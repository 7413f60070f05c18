"""The CPU oracle against the golden vectors and known-answer tests (CPU only).

The golden vectors are an independent float64 restatement of the reference
formulas (tests/golden/make_golden.py); the KATs follow closed forms read off
the reference sources (cited per test).
"""
import math

import numpy as np
import pytest

from util import f16_ulps, max_rel_err, staged_encoder

F16 = np.float16


def test_fp16_conversion_matches_numpy(oracle):
    vals = np.array([0.0, -0.0, 1e-8, 6.1e-5, 0.1, 1.0 / 3, 65504.0, 70000.0, -2.5e-3],
                    np.float32)
    L = oracle.lib()
    got = np.array([L.so_float_to_half(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):  # 70000 rounds to +inf on purpose
        ref = vals.astype(F16)
    assert (got == ref.view(np.uint16)).all()
    back = np.array([L.so_half_to_float(int(h)) for h in got], np.float32)
    assert np.array_equal(back, got.view(F16).astype(np.float32), equal_nan=True)


def test_generators_deterministic_and_distributed(oracle):
    a = oracle.gen_normal(7, 3, (4096,), 0.0, 1.0)
    b = oracle.gen_normal(7, 3, (4096,), 0.0, 1.0)
    c = oracle.gen_normal(7, 4, (4096,), 0.0, 1.0)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    assert not np.array_equal(a, c)
    assert abs(float(a.astype(np.float64).mean())) < 0.06
    assert abs(float(a.astype(np.float64).std()) - 1.0) < 0.05
    u = oracle.gen_u8(7, 5, (1 << 16,))
    assert u.min() == 0 and u.max() == 255
    assert abs(np.bincount(u, minlength=256).std() / 256.0) < 0.2
    p = oracle.gen_palette(7, 6, 32, 0.02)
    assert (np.diff(p.astype(np.float32), axis=1) >= 0).all()
    assert abs(float(p.astype(np.float64).std()) - 0.02) < 0.003
    img = oracle.gen_uniform(7, 8, (10000,), -1.0, 1.0)
    assert img.min() >= -1.0 and img.max() <= 1.0


def test_dequant_golden(oracle, golden):
    # Metal/Dequantize.metal:17-32: out[i] = palette[idx[i]] (bit-exact).
    w = oracle.dequant(golden["dq_idx"], golden["dq_pal"])
    assert np.array_equal(w.view(np.uint16), golden["dq_w"].view(np.uint16))
    # identity-like palette row: P[i] = i - 128
    assert np.array_equal(w[2].astype(np.float32), golden["dq_idx"][2].astype(np.float32) - 128)


@pytest.mark.parametrize("epi,key", [(0, "lin_y_bias"), (1, "lin_y_gelu"), (2, "lin_y_res"),
                                     (3, "lin_y_rope")])
def test_linear_golden(oracle, golden, epi, key):
    y = oracle.linear(golden["lin_x"], golden["lin_idx"], golden["lin_pal"], golden["lin_bias"],
                      epilogue=epi, residual=golden["lin_res"] if epi == 2 else None,
                      rope=golden["lin_table"].astype(np.float32) if epi == 3 else None,
                      rope_period=24, heads=2, head_dim=64)
    # float32 accumulation vs float64: at most one fp16 rounding step apart.
    assert f16_ulps(y, golden[key]) <= 2
    assert max_rel_err(y, golden[key]) < 2e-3


def test_layernorm_golden(oracle, golden):
    y = oracle.layernorm(golden["ln_x"], golden["ln_g"], golden["ln_b"], 1e-6)
    assert f16_ulps(y, golden["ln_y"]) <= 1


def test_rope_table_golden_and_kat(oracle, golden):
    t = oracle.rope_table(4, 6)
    assert np.abs(t - golden["rope_table_4x6"]).max() < 2e-6
    # KATs from Metal/RoPE.metal:22-52. Token 0 = (h 0, w 0): identity rotation.
    assert np.allclose(t[0, :, 0], 1.0) and np.allclose(t[0, :, 1], 0.0)
    # token (h=1, w=2) = 1*6 + 2: pair 0 (x axis, freq 1) has angle 2; pair 16
    # (y axis, freq 1) has angle 1; pair 1 has freq 10000^(-1/16).
    p = 1 * 6 + 2
    assert abs(t[p, 0, 0] - math.cos(2.0)) < 1e-6 and abs(t[p, 0, 1] - math.sin(2.0)) < 1e-6
    assert abs(t[p, 16, 0] - math.cos(1.0)) < 1e-6
    f1 = 10000.0 ** (-1.0 / 16.0)
    assert abs(t[p, 1, 1] - math.sin(2.0 * f1)) < 1e-6
    # every entry is a unit vector (the only property RoPETests.swift:108-113 checks)
    assert np.allclose((t ** 2).sum(-1), 1.0, atol=1e-6)


def test_rope_apply_golden(oracle, golden):
    out = oracle.rope_apply(golden["rope_qkv"], 2, 64, golden["rope_table_4x6"], 24)
    assert f16_ulps(out, golden["rope_out"]) <= 1
    # v third untouched
    assert np.array_equal(out[:, 256:].view(np.uint16), golden["rope_qkv"][:, 256:].view(np.uint16))


def test_attention_golden(oracle, golden):
    o = oracle.attention(golden["att_qkv"], 2, 37, 2, 64)
    assert max_rel_err(o, golden["att_o"]) < 2e-3


def test_attention_kat_zero_query_is_mean_of_v(oracle):
    # q = 0 -> uniform softmax -> output = mean of V (AttentionKernels.swift:48-68).
    seq, heads = 50, 2
    qkv = oracle.gen_normal(3, 9, (seq, 3 * heads * 64))
    qkv[:, :heads * 64] = 0
    o = oracle.attention(qkv, 1, seq, heads, 64)
    v = qkv[:, 2 * heads * 64:].astype(np.float64)
    assert np.abs(o.astype(np.float64) - v.mean(0)).max() < 2e-3


@pytest.mark.parametrize("order", [0, 1])
def test_prune_golden_with_ties(oracle, golden, order):
    feats, _, idx = oracle.prune(golden["pr_x"], 2, 24, 12, norm=0, order=order)
    assert np.array_equal(idx, golden[f"pr_idx_o{order}"])
    assert np.array_equal(feats.view(np.uint16), golden[f"pr_feats_o{order}"].view(np.uint16))


def test_prune_l1_score(oracle, golden):
    _, _, idx = oracle.prune(golden["pr_x"], 2, 24, 12, norm=1, order=0)
    assert np.array_equal(idx, golden["pr_idx_l1"])


def test_prune_gathers_rope_rows(oracle):
    x = oracle.gen_normal(1, 2, (2 * 16, 32))
    table = oracle.rope_table(4, 4)
    feats, rope_out, idx = oracle.prune(x, 2, 16, 5, rope=table, rope_period=16)
    for b in range(2):
        for i in range(5):
            assert np.array_equal(rope_out[b * 5 + i], table[idx[b, i]])


def test_patch_embed_golden(oracle, golden):
    out = oracle.patch_embed(golden["pe_img"], golden["pe_w"], golden["pe_b"], 14)
    assert f16_ulps(out, golden["pe_out"]) <= 2


def test_vit_block_golden(oracle, golden):
    blk = oracle.SyntheticBlock.__new__(oracle.SyntheticBlock)
    dim = 128
    blk.ln1_gamma = blk.ln2_gamma = np.ones(dim, F16)
    blk.ln1_beta = blk.ln2_beta = np.zeros(dim, F16)
    for name in ("qkv", "proj", "fc1", "fc2"):
        setattr(blk, name, {"idx": golden[f"blk_{name}_idx"], "palette": golden[f"blk_{name}_pal"],
                            "bias": golden[f"blk_{name}_bias"]})
    y = oracle.vit_block(golden["blk_x"], 1, 16, 2, blk, golden["blk_table"], 16)
    assert max_rel_err(y, golden["blk_y"]) < 5e-3


def test_encoder_small_end_to_end(oracle):
    # 2 blocks, 8x8 grid, prune after block 1 to 32 tokens: shapes, index order,
    # determinism (same seed -> bit-identical output).
    dim, heads, hidden = 256, 4, 512
    blocks = [oracle.SyntheticBlock(11, i, dim, hidden) for i in range(2)]
    img = oracle.gen_uniform(11, 99, (1, 112, 112, 3), -1.0, 1.0)
    pw = oracle.gen_normal(11, 98, (dim, 3, 14, 14), 0.0, 0.02)
    pb = oracle.gen_normal(11, 97, (dim,), 0.0, 0.02)
    f1, i1 = oracle.encoder_forward(img, blocks, pw, pb, heads=heads, prune_after=1, keep=32)
    f2, i2 = oracle.encoder_forward(img, blocks, pw, pb, heads=heads, prune_after=1, keep=32)
    assert f1.shape == (1, 32, dim) and i1.shape == (1, 32)
    assert (np.diff(i1[0]) > 0).all() and i1.min() >= 0 and i1.max() < 64
    assert np.array_equal(f1.view(np.uint16), f2.view(np.uint16)) and np.array_equal(i1, i2)
    assert np.isfinite(f1.astype(np.float32)).all()


def test_preprocess_rgba_matches_numpy_float32(oracle):
    # (x - mean) / std in float32 with IEEE division, rounded to fp16; alpha
    # dropped; exact values at mean, mean + std, mean - 2 std
    rng = np.random.default_rng(3)
    rgba = rng.random((3, 17, 19, 4), dtype=np.float32)
    mean = np.array([0.485, 0.456, 0.406], np.float32)
    std = np.array([0.229, 0.224, 0.225], np.float32)
    ref = ((rgba[..., :3] - mean) / std).astype(np.float16)
    got = oracle.preprocess_rgba(rgba)
    assert got.shape == (3, 17, 19, 3)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    known = np.zeros((1, 1, 3, 4), np.float32)
    known[0, 0, 0, :3] = mean
    known[0, 0, 1, :3] = mean + std
    known[0, 0, 2, :3] = mean - 2 * std
    known[..., 3] = 0.5
    k = oracle.preprocess_rgba(known).astype(np.float32)[0, 0]
    assert np.allclose(k[0], 0.0, atol=1e-6) and np.allclose(k[1], 1.0, atol=2e-3)
    assert np.allclose(k[2], -2.0, atol=2e-3)


def test_restore_spatial_places_rows_and_zeros(oracle):
    rng = np.random.default_rng(4)
    pruned = rng.standard_normal((2, 5, 8)).astype(np.float16)
    idx = np.stack([rng.permutation(12)[:5] for _ in range(2)]).astype(np.int32)
    out = oracle.restore_spatial(pruned, idx, 12)
    assert out.shape == (2, 12, 8)
    for b in range(2):
        assert np.array_equal(out[b, idx[b]].view(np.uint16), pruned[b].view(np.uint16))
        rest = np.setdiff1d(np.arange(12), idx[b])
        assert not np.any(out[b, rest].astype(np.float32))


def _conv_neck_f64(x, batch, h, w, w1, b1, w2, b2):
    # independent restatement: float64 convolutions, the conv1 output rounded
    # to fp16 as the reference keeps it in an fp16 tensor
    din = x.shape[-1]
    xs = x.astype(np.float64).reshape(batch, h, w, din)
    mid = (np.einsum("bhwc,oc->bhwo", xs, w1.astype(np.float64)) + b1.astype(np.float64))
    mid = mid.astype(np.float16).astype(np.float64)
    pad = np.pad(mid, ((0, 0), (1, 1), (1, 1), (0, 0)))
    out = np.zeros((batch, h, w, w2.shape[0]))
    for ky in range(3):
        for kx in range(3):
            out += np.einsum("bhwc,oc->bhwo", pad[:, ky:ky + h, kx:kx + w],
                             w2[:, :, ky, kx].astype(np.float64))
    return out + b2.astype(np.float64)


def test_neck_matches_float64_convolution(oracle):
    rng = np.random.default_rng(5)
    batch, h, w, din, dout = 2, 5, 6, 64, 32
    x = rng.standard_normal((batch, h * w, din)).astype(np.float16)
    w1 = (rng.standard_normal((dout, din)) * 0.05).astype(np.float16)
    b1 = (rng.standard_normal(dout) * 0.01).astype(np.float16)
    w2 = (rng.standard_normal((dout, dout, 3, 3)) * 0.05).astype(np.float16)
    b2 = (rng.standard_normal(dout) * 0.01).astype(np.float16)
    got = oracle.neck(x, batch, h, w, w1, b1, w2, b2)
    ref = _conv_neck_f64(x, batch, h, w, w1, b1, w2, b2)
    assert got.shape == (batch, h, w, dout)
    assert max_rel_err(got, ref) < 2e-3


# ------------------------------------------------------------------ windowed encoder variant
def _bilinear_weights(n_out, n_in):
    # half-pixel centres, source clamped at 0 and at n_in - 1 (float64)
    w = np.zeros((n_out, n_in))
    for i in range(n_out):
        s = max((i + 0.5) * n_in / n_out - 0.5, 0.0)
        i0 = min(int(np.floor(s)), n_in - 1)
        i1 = min(i0 + 1, n_in - 1)
        f = s - i0
        w[i, i0] += 1.0 - f
        w[i, i1] += f
    return w


def _windowed_inputs(oracle, seed, dim, hidden, nblocks, pos_grid, image=112, batch=1):
    blocks = [oracle.SyntheticBlock(seed, i, dim, hidden) for i in range(nblocks)]
    pw = oracle.gen_normal(seed, 900, (dim, 3, 14, 14), 0.0, 0.02)
    pb = oracle.gen_normal(seed, 901, (dim,), 0.0, 0.02)
    cls = oracle.gen_normal(seed, 902, (dim,), 0.0, 0.5)
    pos = oracle.gen_normal(seed, 903, (1 + pos_grid * pos_grid, dim), 0.0, 0.5)
    img = oracle.gen_uniform(seed, 904, (batch, image, image, 3), -1.0, 1.0)
    return blocks, pw, pb, cls, pos, img


def test_windowed_encoder_embedding_matches_float64_resize(oracle):
    # no blocks: out = fp16(patch token + fp16(bilinear resize of the grid
    # positions)); the resize against a float64 separable restatement
    dim, grid, pg = 64, 8, 3
    _, pw, pb, cls, pos, img = _windowed_inputs(oracle, 61, dim, 128, 0, pg, batch=2)
    out = oracle.windowed_encoder_forward(img, [], pw, pb, cls, pos, heads=1, window=4)
    tok = oracle.patch_embed(img, pw, pb).astype(np.float64).reshape(2, grid * grid, dim)
    wy = _bilinear_weights(grid, pg)
    up = np.einsum("yi,xj,ijc->yxc", wy, wy, pos[1:].astype(np.float64).reshape(pg, pg, dim))
    up16 = up.reshape(grid * grid, dim).astype(np.float16).astype(np.float64)
    ref = (tok + up16[None]).astype(np.float16)
    assert out.shape == (2, grid * grid, dim)
    assert f16_ulps(out, ref) <= 1
    # pos_grid == grid: the resize is the identity, the sum exact
    pos8 = oracle.gen_normal(62, 1, (1 + grid * grid, dim), 0.0, 0.5)
    out8 = oracle.windowed_encoder_forward(img, [], pw, pb, None, pos8, heads=1, window=4)
    ref8 = (tok + pos8[1:].astype(np.float64)[None]).astype(np.float16)
    assert np.array_equal(out8.view(np.uint16), ref8.view(np.uint16))


def test_windowed_encoder_matches_window_partition_composition(oracle):
    # 8 blocks on an 8x8 grid with 4x4 windows: blocks 1, 3, 5, 7 global, the
    # others windowed. Independent composition from the oracle's operators with
    # the reference's reshape/transpose window partition; bit-identical.
    dim, heads, hidden, nb, pg, grid = 128, 2, 256, 8, 4, 8
    blocks, pw, pb, cls, pos, img = _windowed_inputs(oracle, 63, dim, hidden, nb, pg)
    got = oracle.windowed_encoder_forward(img, blocks, pw, pb, cls, pos, heads=heads)

    S, T, win = grid * grid, grid * grid + 1, pg
    zero = oracle.windowed_encoder_forward(img, [], pw, pb, cls, pos, heads=heads)[0]
    x = np.concatenate([(cls.astype(np.float32) + pos[0].astype(np.float32)).astype(np.float16)[None],
                        zero], axis=0)
    table = np.concatenate([np.stack([np.ones(32), np.zeros(32)], -1)[None].astype(np.float32),
                            oracle.rope_table(grid, grid)], axis=0)
    stride = max(1, nb // 4)
    global_blocks = set(range(stride - 1, nb, stride))
    assert global_blocks == {1, 3, 5, 7}
    P = grid // win

    def partition(a):  # [S, C] grid order -> [P*P*win*win, C] window-major
        c = a.shape[-1]
        return a.reshape(P, win, P, win, c).transpose(0, 2, 1, 3, 4).reshape(S, c)

    def reverse(a):
        c = a.shape[-1]
        return a.reshape(P, P, win, win, c).transpose(0, 2, 1, 3, 4).reshape(S, c)

    for i, blk in enumerate(blocks):
        ln = oracle.layernorm(x)
        qkv = oracle.linear(ln, **_lin(blk.qkv), epilogue=oracle.EPI_BIAS_ROPE_QKV, rope=table,
                            rope_period=T, heads=heads)
        if i in global_blocks:
            att = oracle.attention(qkv, 1, T, heads, 64)
        else:
            wins = oracle.attention(partition(qkv[1:]), P * P, win * win, heads, 64)
            att = np.concatenate([np.zeros((1, dim), np.float16), reverse(wins)], axis=0)
        x = oracle.linear(att, **_lin(blk.proj), epilogue=oracle.EPI_BIAS_RESIDUAL, residual=x,
                          heads=heads)
        h = oracle.linear(oracle.layernorm(x), **_lin(blk.fc1), epilogue=oracle.EPI_BIAS_GELU,
                          heads=heads)
        x = oracle.linear(h, **_lin(blk.fc2), epilogue=oracle.EPI_BIAS_RESIDUAL, residual=x,
                          heads=heads)
    assert got.shape == (1, S, dim)
    assert np.array_equal(got[0].view(np.uint16), x[1:].view(np.uint16))


def _lin(d):
    return {"idx": d["idx"], "palette": d["palette"], "bias": d["bias"]}


@pytest.mark.parametrize("keep", [1, 5, 16])
@pytest.mark.parametrize("order", [0, 1])
def test_prune_keep_extremes_known_answer(oracle, keep, order):
    # rows of constant value v (distinct |v| per row, exact in fp16): the L2
    # score ranks rows by |v|; keep 1 is the arg-max, keep = seq keeps every
    # row (index order: 0..seq-1; score order: by descending score)
    seq, d = 16, 8
    rng = np.random.default_rng(keep * 10 + order)
    x = np.empty((2 * seq, d), F16)
    for b in range(2):
        v = rng.permutation(np.arange(1, seq + 1)) * rng.choice([-1, 1], seq)
        x[b * seq:(b + 1) * seq] = v[:, None].astype(F16)
    feats, _, idx = oracle.prune(x, 2, seq, keep, norm=0, order=order)
    for b in range(2):
        mag = np.abs(x[b * seq:(b + 1) * seq, 0].astype(np.float64))
        top = np.argsort(-mag, kind="stable")[:keep]
        want = top if order == 1 else np.sort(top)
        assert np.array_equal(idx[b], want)
        assert np.array_equal(feats[b * keep:(b + 1) * keep].view(np.uint16),
                              x[b * seq + want].view(np.uint16))


# ------------------------------------------------------------------ reference rounding points
def _graph_ops_numpy(h0, bias, epi, residual=None, table=None, heads=2, head_dim=8):
    """numpy restatement of the reference's fp16 graph ops after the matmul:
    every op on fp16 operands is computed in float32 and rounded to fp16
    (numpy's float16 arithmetic), as MPSGraph returns an fp16 tensor per op.
    MPSAttention.swift:113-160 (bias, RoPE with cos/sin cast to fp16) and
    ViTEncoder.swift:559-605 (residual) / :581-589 (GELU)."""
    from scipy.special import erf
    r = (h0 + bias.astype(F16)).astype(F16)
    if epi == 1:
        sqrt2 = F16(1.41421356)
        div = (r / sqrt2).astype(F16)
        e = erf(div.astype(np.float64)).astype(F16)
        return ((F16(0.5) * r).astype(F16) * (F16(1.0) + e).astype(F16)).astype(F16)
    if epi == 2:
        return (residual.astype(F16) + r).astype(F16)
    if epi == 3:
        out = r.copy()
        qk = 2 * heads * head_dim
        for i in range(r.shape[0]):
            t = table[i % table.shape[0]].astype(F16)  # [head_dim/2, 2], cast to fp16
            for j in range(0, qk, 2):
                p = (j % head_dim) // 2
                c, s = t[p, 0], t[p, 1]
                a, b = r[i, j], r[i, j + 1]
                out[i, j] = F16(F16(a * c) - F16(b * s))
                out[i, j + 1] = F16(F16(a * s) + F16(b * c))
        return out
    return r


@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_graph_rounding_linear_matches_numpy(oracle, epi):
    # The matmul result rounded to fp16 comes from the oracle itself (graph
    # mode, no bias), so the comparison covers the ops after it bit for bit.
    m, k, heads, hd = 24, 64, 2, 8
    n = 3 * heads * hd
    x = oracle.gen_normal(81, 1, (m, k))
    idx = oracle.gen_u8(81, 2, (n, k))
    pal = oracle.gen_palette(81, 3, n, 0.2)
    bias = oracle.gen_normal(81, 4, (n,), 0.0, 0.5)
    res = oracle.gen_normal(81, 5, (m, n))
    table = oracle.rope_table(4, 6, hd)
    with oracle.rounding(oracle.ROUND_GRAPH):
        h0 = oracle.linear(x, idx, pal, None, epilogue=0)
        got = oracle.linear(x, idx, pal, bias, epilogue=epi,
                            residual=res if epi == 2 else None,
                            rope=table if epi == 3 else None, rope_period=24,
                            heads=heads, head_dim=hd)
    ref = _graph_ops_numpy(h0, bias, epi, res, table, heads, hd)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    # the mode is restored on exit, and the two modes agree within the spec
    assert oracle.lib().so_rounding() == oracle.ROUND_FUSED
    fused = oracle.linear(x, idx, pal, bias, epilogue=epi, residual=res if epi == 2 else None,
                          rope=table if epi == 3 else None, rope_period=24, heads=heads,
                          head_dim=hd)
    assert max_rel_err(got, fused) < 1e-2


def test_graph_rounding_layernorm_matches_numpy(oracle):
    # ViTEncoder.swift:466-474: mean, variance about the fp16 mean, centre,
    # sqrt(var + eps), divide, scale, shift, each an fp16 tensor
    x = oracle.gen_normal(82, 1, (16, 256), 0.3, 2.0)
    g = oracle.gen_normal(82, 2, (256,), 1.0, 0.1)
    b = oracle.gen_normal(82, 3, (256,), 0.0, 0.1)
    with oracle.rounding(oracle.ROUND_GRAPH):
        got = oracle.layernorm(x, g, b, 1e-6)
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1, keepdims=True).astype(np.float32).astype(F16)
    var = ((xd - mean.astype(np.float64)) ** 2).mean(axis=1, keepdims=True).astype(
        np.float32).astype(F16)
    denom = np.sqrt((var + F16(1e-6)).astype(F16)).astype(F16)
    cen = (x - mean).astype(F16)
    ref = ((cen / denom).astype(F16) * g).astype(F16) + b
    assert np.array_equal(got.view(np.uint16), ref.astype(F16).view(np.uint16))
    fused = oracle.layernorm(x, g, b, 1e-6)
    assert max_rel_err(got, fused) < 1e-2


def test_staged_oracle_equals_encoder_forward(oracle):
    # small shape: the staged composition used above is the oracle's encoder
    blocks = [oracle.SyntheticBlock(55, i, 256, 512) for i in range(3)]
    pw = oracle.gen_normal(55, 900, (256, 3, 14, 14), 0.0, 0.02)
    pb = oracle.gen_normal(55, 901, (256,), 0.0, 0.02)
    img = oracle.gen_uniform(55, 77, (1, 112, 112, 3), -1.0, 1.0)
    _, f, i = staged_encoder(oracle, img, blocks, pw, pb, prune_after=2, keep=32)
    ef, ei = oracle.encoder_forward(img, blocks, pw, pb, heads=4, prune_after=2, keep=32)
    assert np.array_equal(i, ei[0]) and np.array_equal(f.view(np.uint16), ef[0].view(np.uint16))
