"""Generate tests/golden/*.npz: small golden vectors for the encoder hot path.

The reference (Swift + Metal + MPSGraph, OrdoSAM3Sensor/Sources/Sam3Sensor)
cannot run on this platform and its tests hold no golden vectors for this
path, so these vectors come from an independent float64 numpy restatement of
the reference formulas, written separately from the C++ oracle:

  dequant    W[n,k] = P[n, idx[n,k]]                  Metal/Dequantize.metal:17-32
  linear     y = x W^T + b (+GELU | +residual | +RoPE) MPSAttention.swift:113-183,
                                                      ViTEncoder.swift:979-997
  layernorm  (x - mean)/sqrt(var + eps) g + b          ViTEncoder.swift:822-831
  rope       table + interleaved-pair rotation         Metal/RoPE.metal:22-52,
                                                      MPSAttention.swift:137-160
  attention  softmax(q k^T / sqrt(d)) v                AttentionKernels.swift:48-68
  prune      score, top-k (ties -> lower index), gather TokenPruner.swift:32-126
  patch      14x14 stride-14 conv, tokens h*W + w      ViTEncoder.swift:218-263,
                                                      Metal/ViTUtils.metal:53-76
  block      LN1-QKV-RoPE-SDPA-proj-res-LN2-fc1-GELU-fc2-res ViTEncoder.swift:457-615

Inputs are fp16 (seeded numpy); outputs are float64 results rounded once to
fp16 at the same tensor boundaries the oracle and the CUDA path use.
Run:  python tests/golden/make_golden.py   (writes next to this file)
"""
from __future__ import annotations

import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F16 = np.float16


def f64(a):
    return np.asarray(a, dtype=np.float64)


def erf(x):
    return np.vectorize(math.erf)(x)


def gelu(x):
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def palette_rows(rng, n, std=0.02):
    p = rng.normal(0.0, std, size=(n, 256)).astype(F16)
    return np.sort(p.astype(np.float32), axis=1).astype(F16)


def rope_table(gh, gw, hd=64, theta=10000.0):
    q = hd // 4
    t = np.zeros((gh * gw, hd // 2, 2))
    for p in range(gh * gw):
        h, w = divmod(p, gw)
        for i in range(q):
            freq = 1.0 / theta ** (2 * i / (2 * q))
            t[p, i] = (math.cos(w * freq), math.sin(w * freq))
            t[p, q + i] = (math.cos(h * freq), math.sin(h * freq))
    return t


def rope_rotate(y, table, rows, heads, hd):
    """Rotate interleaved pairs of the q and k thirds of packed rows y (float64)."""
    y = y.copy()
    dim = heads * hd
    for i in range(y.shape[0]):
        t = table[i % rows]
        for c in range(0, 2 * dim, 2):
            j = (c % hd) // 2
            cs, sn = t[j]
            a, b = y[i, c], y[i, c + 1]
            y[i, c], y[i, c + 1] = a * cs - b * sn, a * sn + b * cs
    return y


def linear(x, idx, pal, bias):
    w = f64(pal[np.arange(idx.shape[0])[:, None], idx])
    return f64(x) @ w.T + f64(bias)


def layernorm(x, eps=1e-6, g=None, b=None):
    x = f64(x)
    mu = x.mean(1, keepdims=True)
    var = ((x - mu) ** 2).mean(1, keepdims=True)
    y = (x - mu) / np.sqrt(var + eps)
    if g is not None:
        y = y * f64(g)
    if b is not None:
        y = y + f64(b)
    return y


def attention(qkv, batch, seq, heads, hd):
    q = f64(qkv).reshape(batch, seq, 3, heads, hd)
    o = np.zeros((batch, seq, heads, hd))
    for b in range(batch):
        for h in range(heads):
            s = q[b, :, 0, h] @ q[b, :, 1, h].T / math.sqrt(hd)
            p = np.exp(s - s.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            o[b, :, h] = p @ q[b, :, 2, h]
    return o.reshape(batch * seq, heads * hd)


def topk(scores, keep, order):
    idx = sorted(range(len(scores)), key=lambda i: (-scores[i], i))[:keep]
    return sorted(idx) if order == 0 else idx


def block(x, batch, seq, heads, w, table, rows):
    hd = 64
    dim = heads * hd
    ln1 = layernorm(x).astype(F16)
    qkv = rope_rotate(linear(ln1, *w["qkv"]), table, rows, heads, hd).astype(F16)
    att = attention(qkv, batch, seq, heads, hd).astype(F16)
    x1 = (linear(att, *w["proj"]) + f64(x)).astype(F16)
    ln2 = layernorm(x1).astype(F16)
    h = gelu(linear(ln2, *w["fc1"])).astype(F16)
    return (linear(h, *w["fc2"]) + f64(x1)).astype(F16)


def block_weights(rng, dim, hidden):
    def lin(n, k):
        return (rng.integers(0, 256, size=(n, k), dtype=np.uint8), palette_rows(rng, n),
                rng.normal(0, 0.01, size=n).astype(F16))
    return {"qkv": lin(3 * dim, dim), "proj": lin(dim, dim), "fc1": lin(hidden, dim),
            "fc2": lin(dim, hidden)}


def flat_weights(prefix, w):
    out = {}
    for name, (idx, pal, bias) in w.items():
        out[f"{prefix}{name}_idx"] = idx
        out[f"{prefix}{name}_pal"] = pal
        out[f"{prefix}{name}_bias"] = bias
    return out


def main():
    rng = np.random.default_rng(20240601)
    g = {}

    # dequant (hand-built rows + random rows)
    idx = rng.integers(0, 256, size=(8, 64), dtype=np.uint8)
    idx[0] = np.arange(64)
    idx[1] = 255 - np.arange(64)
    pal = palette_rows(rng, 8)
    pal[2] = (np.arange(256) - 128).astype(F16)  # identity-like palette P[i] = i - 128
    g["dq_idx"], g["dq_pal"], g["dq_w"] = idx, pal, pal[np.arange(8)[:, None], idx]

    # linear with each epilogue; heads=2 x 64 for the RoPE case (n = 384)
    m, k, n = 48, 128, 384
    x = rng.normal(0, 1, size=(m, k)).astype(F16)
    li = rng.integers(0, 256, size=(n, k), dtype=np.uint8)
    lp = palette_rows(rng, n)
    lb = rng.normal(0, 0.01, size=n).astype(F16)
    res = rng.normal(0, 1, size=(m, n)).astype(F16)
    table = rope_table(4, 6)
    acc = linear(x, li, lp, lb)
    g.update(lin_x=x, lin_idx=li, lin_pal=lp, lin_bias=lb, lin_res=res, lin_table=table)
    g["lin_y_bias"] = acc.astype(F16)
    g["lin_y_gelu"] = gelu(acc).astype(F16)
    g["lin_y_res"] = (acc + f64(res)).astype(F16)
    g["lin_y_rope"] = rope_rotate(acc, table, 24, 2, 64).astype(F16)

    # layernorm with gamma/beta
    lx = (rng.normal(0, 2, size=(16, 256)) + 0.5).astype(F16)
    lg = rng.normal(1, 0.1, size=256).astype(F16)
    lbb = rng.normal(0, 0.1, size=256).astype(F16)
    g.update(ln_x=lx, ln_g=lg, ln_b=lbb, ln_y=layernorm(lx, 1e-6, lg, lbb).astype(F16))

    # RoPE table (non-square grid) and stand-alone rotation of packed rows
    g["rope_table_4x6"] = table.astype(np.float32)
    rq = rng.normal(0, 1, size=(24, 3 * 128)).astype(F16)
    g["rope_qkv"] = rq
    g["rope_out"] = rope_rotate(f64(rq), table, 24, 2, 64).astype(F16)

    # attention: batch 2, seq 37 (ragged vs 64-key tiles), 2 heads
    aq = rng.normal(0, 1, size=(2 * 37, 3 * 128)).astype(F16)
    g["att_qkv"] = aq
    g["att_o"] = attention(aq, 2, 37, 2, 64).astype(F16)

    # prune: batch 2, seq 24, d 16; image 1 has deliberate score ties
    # Image 1: ten clear winners, rows 3/7/11/20 tied exactly (20 = -7) and
    # competing for the last two of the 12 slots -> rows 3 and 7 must win.
    px = rng.normal(0, 1, size=(2 * 24, 16))
    px[24:] *= 0.2
    px[24 + np.array([0, 1, 2, 5, 6, 8, 9, 10, 12, 13])] *= 15.0
    tie = rng.normal(0, 1, size=16)
    px[24 + 3] = px[24 + 7] = px[24 + 11] = tie
    px[24 + 20] = -tie
    px = px.astype(F16)
    scores = np.sqrt((f64(px) ** 2).sum(1))
    g["pr_x"] = px
    g["pr_scores"] = scores.astype(np.float32)
    for order in (0, 1):
        ids = np.array([topk(scores[b * 24:(b + 1) * 24], 12, order) for b in range(2)],
                       dtype=np.int32)
        g[f"pr_idx_o{order}"] = ids
        g[f"pr_feats_o{order}"] = np.concatenate([px[b * 24 + ids[b]] for b in range(2)])
    l1 = np.abs(f64(px)).sum(1)
    g["pr_idx_l1"] = np.array([topk(l1[b * 24:(b + 1) * 24], 12, 0) for b in range(2)],
                              dtype=np.int32)

    # patch embedding: 1 x 28 x 28 x 3 image, dim 128
    img = rng.uniform(-1, 1, size=(1, 28, 28, 3)).astype(F16)
    pw = rng.normal(0, 0.02, size=(128, 3, 14, 14)).astype(F16)
    pb = rng.normal(0, 0.02, size=128).astype(F16)
    cols = np.zeros((4, 588))
    for p in range(4):
        py, pxx = divmod(p, 2)
        patch = f64(img[0, py * 14:(py + 1) * 14, pxx * 14:(pxx + 1) * 14, :])  # [ky, kx, c]
        cols[p] = patch.transpose(2, 0, 1).reshape(-1)
    g.update(pe_img=img, pe_w=pw, pe_b=pb,
             pe_out=(cols @ f64(pw).reshape(128, -1).T + f64(pb)).astype(F16))

    # one ViT block: dim 128 (2 heads), hidden 256, 4x4 grid, batch 1
    dim, hidden, heads = 128, 256, 2
    bw = block_weights(rng, dim, hidden)
    bx = rng.normal(0, 1, size=(16, dim)).astype(F16)
    bt = rope_table(4, 4)
    g.update(flat_weights("blk_", bw))
    g["blk_x"], g["blk_table"] = bx, bt.astype(np.float32)
    g["blk_y"] = block(bx, 1, 16, heads, bw, bt, 16)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **g)
    print("wrote", os.path.join(HERE, "golden.npz"), len(g), "arrays")


if __name__ == "__main__":
    main()
