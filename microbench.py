#!/usr/bin/env python
"""Kernel micro-benchmarks for libsam3cuda (one operator, one shape).

    python microbench.py gemm --m 41472 --n 4096 --k 1024 --epi gelu
    python microbench.py attention --batch 8 --seq 5184
    python microbench.py layernorm --m 41472
    python microbench.py prune --batch 16        (L2 score + top-2592 + gather of rows and RoPE rows)
    python microbench.py patch --batch 8 [--rgba]
    python microbench.py preprocess --batch 8
    python microbench.py neck --batch 8          (restoreSpatial + neck, 72x72, 1024 -> 256)
    python microbench.py windowed --batch 8      (checkpoint-faithful encoder, 32 blocks, 1008^2)
    python microbench.py encoder --batch 8 [--blocks 32]  (pruned encoder, device buffers)

Inputs are synthetic device tensors (torch is used only to allocate and fill
them); each iteration calls the operator through the C ABI; timings are CUDA
events on the library's stream around each launch (sam3_profile_*), after
warm-up. Prints one JSON line per operator.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "metal-sam-ios-experiments_b200"))

EPIS = {"bias": 0, "gelu": 1, "residual": 2, "rope": 3}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"])
    except Exception:
        return 1590.0, 6650.0


def main():
    import torch
    import sam3cuda as sam3

    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=("gemm", "attention", "layernorm", "prune", "dequant", "patch",
                                   "preprocess", "neck", "windowed", "encoder"))
    ap.add_argument("--rgba", action="store_true",
                    help="patch: f32 RGBA frames, normalisation fused into the patch gather")
    ap.add_argument("--m", type=int, default=41472)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--epi", choices=tuple(EPIS), default="bias")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=5184)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--hidden", type=int, default=4096, help="windowed: MLP width (checkpoint 4736)")
    ap.add_argument("--blocks", type=int, default=32, help="encoder: blocks (pruned after half)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()

    dev = torch.device("cuda", 0)
    ctx = sam3.Context(0, max_batch=1)
    tf_peak, bw_peak = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(0)

    def run(fn):
        torch.cuda.synchronize()  # inputs are filled on torch's stream, the operator runs on ctx's
        for _ in range(a.warmup):
            fn()
        ctx.sync()
        ctx.profile_enable(True)
        for _ in range(a.iters):
            fn()
        prof = ctx.profile_read()
        ctx.profile_enable(False)
        return prof

    if a.op in ("gemm", "dequant"):
        x = torch.randn((a.m, a.k), generator=g, device=dev).half()
        idx = torch.randint(0, 256, (a.n, a.k), generator=g, device=dev, dtype=torch.uint8)
        pal = (torch.randn((a.n, 256), generator=g, device=dev) * 0.02).half().sort(dim=1).values
        bias = (torch.randn((a.n,), generator=g, device=dev) * 0.01).half()
        y = torch.empty((a.m, a.n), dtype=torch.float16, device=dev)
        w = sam3.palette_linear(idx, pal.contiguous(), bias, a.n, a.k)
        if a.op == "dequant":
            out = torch.empty((a.n, a.k), dtype=torch.float16, device=dev)
            prof = run(lambda: ctx.dequant_palette(w, out))["other"]
            ms = prof["ms"] / prof["launches"]
            print(json.dumps({"op": "dequant", "n": a.n, "k": a.k, "us": ms * 1e3,
                              "gbs": prof["bytes"] / prof["launches"] / (ms * 1e-3) / 1e9,
                              "frac_hbm": prof["bytes"] / prof["launches"] / (ms * 1e-3) / 1e9 / bw_peak}))
            return
        epi = EPIS[a.epi]
        res = torch.randn((a.m, a.n), generator=g, device=dev).half() if epi == 2 else None
        rope = None
        rows = 0
        if epi == 3:
            rows = a.seq
            rope = torch.empty((rows, 32, 2), dtype=torch.float32, device=dev)
            side = int(round(rows ** 0.5))
            ctx.rope_table(side, rows // side, 64, 10000.0, rope)
        prof = run(lambda: ctx.linear_palette(x, a.m, w, epi, y, res, rope, rows))["gemm"]
        ms = prof["ms"] / prof["launches"]
        tf = prof["flops"] / prof["launches"] / (ms * 1e-3) / 1e12
        print(json.dumps({"op": "gemm", "m": a.m, "n": a.n, "k": a.k, "epi": a.epi, "us": ms * 1e3,
                          "tflops": tf, "frac_burst_peak": tf / tf_peak}))
    elif a.op == "attention":
        qkv = torch.randn((a.batch * a.seq, 3 * a.heads * 64), generator=g, device=dev).half()
        o = torch.empty((a.batch * a.seq, a.heads * 64), dtype=torch.float16, device=dev)
        prof = run(lambda: ctx.attention(qkv, a.batch, a.seq, a.heads, 64, 0.125, o))["attention"]
        ms = prof["ms"] / prof["launches"]
        tf = prof["flops"] / prof["launches"] / (ms * 1e-3) / 1e12
        print(json.dumps({"op": "attention", "batch": a.batch, "seq": a.seq, "heads": a.heads,
                          "us": ms * 1e3, "tflops": tf, "frac_burst_peak": tf / tf_peak}))
    elif a.op == "neck":
        ctx.close()
        ctx = sam3.Context(0, max_batch=a.batch)
        grid, keep, din, dout = 72, 2592, 1024, 256
        seq = grid * grid
        pruned = torch.randn((a.batch, keep, din), generator=g, device=dev).half()
        idx = torch.stack([torch.randperm(seq, generator=torch.Generator().manual_seed(b))[:keep]
                           .sort().values for b in range(a.batch)]).int().to(dev)
        spatial = torch.empty((a.batch, seq, din), dtype=torch.float16, device=dev)
        w1 = (torch.randn((dout, din), generator=g, device=dev) * 0.03).half()
        b1 = (torch.randn((dout,), generator=g, device=dev) * 0.01).half()
        w2 = (torch.randn((dout, dout, 3, 3), generator=g, device=dev) * 0.03).half()
        b2 = (torch.randn((dout,), generator=g, device=dev) * 0.01).half()
        nw = sam3.neck_weights(w1, b1, w2, b2, din, dout)
        out = torch.empty((a.batch, grid, grid, dout), dtype=torch.float16, device=dev)

        def call():
            ctx.restore_spatial(pruned, idx, a.batch, keep, seq, din, spatial)
            ctx.neck(spatial, a.batch, grid, grid, nw, out)

        prof = run(call)["other"]
        calls = a.iters
        flops = 2.0 * a.batch * seq * dout * (din + 9 * dout)
        ms = prof["ms"] / calls
        print(json.dumps({"op": "neck", "batch": a.batch, "us_per_call": ms * 1e3,
                          "tflops_convs": flops / (ms * 1e-3) / 1e12}))
        ctx.close()
        return
    elif a.op == "encoder":
        sys.path.insert(0, ROOT)
        import bench  # the benchmark's synthetic weights
        ctx.close()
        prune_after = a.blocks // 2 if a.blocks > 1 else 0
        ctx = sam3.Context(0, max_batch=a.batch, num_blocks=a.blocks,
                           prune_after_block=prune_after)
        bench.BLOCKS = a.blocks
        w = bench.make_weights(torch, sam3, dev, 1234)
        img = (torch.rand((a.batch, 1008, 1008, 3), generator=g, device=dev) * 2 - 1).half()
        keep = ctx.out_tokens
        feats = torch.empty((a.batch, keep, 1024), dtype=torch.float16, device=dev)
        idx = torch.empty((a.batch, keep), dtype=torch.int32, device=dev)
        fn = lambda: ctx.encoder_forward(img, a.batch, w, feats, idx)
        prof = run(fn)
        stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.sync()
        ev0.record(stream)
        for _ in range(a.iters):
            fn()
        ev1.record(stream)
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1) / a.iters
        print(json.dumps({
            "op": "encoder", "batch": a.batch, "blocks": a.blocks, "ms_per_call": ms,
            "images_per_s": a.batch / (ms * 1e-3),
            "gemm_tflops": prof["gemm"]["flops"] / (prof["gemm"]["ms"] * 1e-3) / 1e12,
            "attention_tflops": prof["attention"]["flops"] / (prof["attention"]["ms"] * 1e-3) / 1e12}))
        ctx.close()
        return
    elif a.op == "windowed":
        ctx.close()
        ctx = sam3.Context(0, max_batch=a.batch, mlp_hidden=a.hidden)
        dim, hidden, nblocks, pg, size = 1024, a.hidden, 32, 24, 1008
        keep = []

        def t(x):
            keep.append(x)
            return x

        def lin(n, k):
            idx = t(torch.randint(0, 256, (n, k), generator=g, device=dev, dtype=torch.uint8))
            pal = t((torch.randn((n, 256), generator=g, device=dev) * 0.02).half().sort(dim=1)
                    .values.contiguous())
            bias = t((torch.randn((n,), generator=g, device=dev) * 0.01).half())
            return sam3.palette_linear(idx, pal, bias, n, k)

        ones = t(torch.ones(dim, dtype=torch.float16, device=dev))
        zeros = t(torch.zeros(dim, dtype=torch.float16, device=dev))
        blocks = [sam3.block_weights(ones, zeros, lin(3 * dim, dim), lin(dim, dim), ones, zeros,
                                     lin(hidden, dim), lin(dim, hidden)) for _ in range(nblocks)]
        pw = t((torch.randn((dim, 3, 14, 14), generator=g, device=dev) * 0.02).half())
        pb = t((torch.randn((dim,), generator=g, device=dev) * 0.02).half())
        cls = t((torch.randn((dim,), generator=g, device=dev) * 0.02).half())
        pos = t((torch.randn((1 + pg * pg, dim), generator=g, device=dev) * 0.02).half())
        w = sam3.windowed_encoder_weights(pw, pb, cls, pos, pg, blocks)
        img = (torch.rand((a.batch, size, size, 3), generator=g, device=dev) * 2 - 1).half()
        out = torch.empty((a.batch, 5184, dim), dtype=torch.float16, device=dev)
        fn = lambda: ctx.windowed_encoder_forward(img, a.batch, w, out)
        prof = run(fn)
        stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.sync()
        ev0.record(stream)
        for _ in range(a.iters):
            fn()
        ev1.record(stream)
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1) / a.iters
        T = 5185
        win_att = 4.0 * 9 * 576 * 576 * 64 * 16
        glob_att = 4.0 * T * T * 64 * 16
        flops = a.batch * (nblocks * 2.0 * T * dim * (4 * dim + 2 * hidden)
                           + 24 * win_att + 8 * glob_att)
        print(json.dumps({
            "op": "windowed", "batch": a.batch, "hidden": hidden, "ms_per_call": ms, "images_per_s": a.batch / (ms * 1e-3),
            "tflops": flops / (ms * 1e-3) / 1e12,
            "classes_ms_per_call": {k: v["ms"] / a.iters for k, v in prof.items() if v["launches"]},
            "gemm_tflops": prof["gemm"]["flops"] / (prof["gemm"]["ms"] * 1e-3) / 1e12,
            "attention_tflops": prof["attention"]["flops"] / (prof["attention"]["ms"] * 1e-3) / 1e12}))
        ctx.close()
        return
    elif a.op in ("patch", "preprocess"):
        size = 1008
        ctx.close()
        ctx = sam3.Context(0, max_batch=a.batch)
        rgba = torch.rand((a.batch, size, size, 4), generator=g, device=dev)
        rgb = (torch.rand((a.batch, size, size, 3), generator=g, device=dev) * 2 - 1).half()
        if a.op == "preprocess":
            out = torch.empty((a.batch, size, size, 3), dtype=torch.float16, device=dev)
            prof = run(lambda: ctx.preprocess_rgba(rgba, a.batch, size, size, out))["patch"]
            ms = prof["ms"] / prof["launches"]
            gbs = prof["bytes"] / prof["launches"] / (ms * 1e-3) / 1e9
            print(json.dumps({"op": "preprocess", "batch": a.batch, "us": ms * 1e3, "gbs": gbs,
                              "frac_hbm": gbs / bw_peak}))
            return
        pw = (torch.randn((1024, 3, 14, 14), generator=g, device=dev) * 0.02).half()
        pb = (torch.randn((1024,), generator=g, device=dev) * 0.02).half()
        tokens = a.batch * (size // 14) ** 2
        out = torch.empty((tokens, 1024), dtype=torch.float16, device=dev)
        if a.rgba:
            fn = lambda: ctx.patch_embed_rgba(rgba, a.batch, size, size, pw, pb, 14, 1024, out)
        else:
            fn = lambda: ctx.patch_embed(rgb, a.batch, size, size, pw, pb, 14, 1024, out)
        prof = run(fn)["patch"]
        ms = prof["ms"] / prof["launches"] * 3  # im2col, weight pad and GEMM per call
        print(json.dumps({"op": "patch", "rgba": a.rgba, "batch": a.batch, "us_per_call": ms * 1e3,
                          "gbs_gather_and_pad": prof["bytes"] / (prof["ms"] * 1e-3) / 1e9}))
        ctx.close()
        return
    elif a.op == "prune":
        # the encoder's prune after block 16: seq tokens per image -> seq / 2,
        # L2 score, kept in token order, with their RoPE rows
        ctx.close()
        ctx = sam3.Context(0, max_batch=a.batch)
        keep = a.seq // 2
        x = torch.randn((a.batch * a.seq, 1024), generator=g, device=dev).half()
        rope = torch.randn((a.seq, 64), generator=g, device=dev)
        feats = torch.empty((a.batch * keep, 1024), dtype=torch.float16, device=dev)
        rope_out = torch.empty((a.batch * keep, 64), dtype=torch.float32, device=dev)
        idx = torch.empty((a.batch, keep), dtype=torch.int32, device=dev)
        prof = run(lambda: ctx.prune(x, a.batch, a.seq, 1024, keep, sam3.SCORE_L2,
                                     sam3.ORDER_INDEX, feats, idx, rope, a.seq, 64,
                                     rope_out))["prune"]
        calls = prof["launches"] / 3  # score, select, gather per call
        us = prof["ms"] / calls * 1e3
        gbs = prof["bytes"] / (prof["ms"] * 1e-3) / 1e9
        print(json.dumps({"op": "prune", "batch": a.batch, "seq": a.seq, "keep": keep,
                          "us_per_call": us, "gbs": gbs, "frac_hbm": gbs / bw_peak}))
    else:
        x = torch.randn((a.m, 1024), generator=g, device=dev).half()
        y = torch.empty_like(x)
        prof = run(lambda: ctx.layernorm(x, a.m, 1024, None, None, 1e-6, y))["layernorm"]
        ms = prof["ms"] / prof["launches"]
        gbs = prof["bytes"] / prof["launches"] / (ms * 1e-3) / 1e9
        print(json.dumps({"op": "layernorm", "m": a.m, "us": ms * 1e3, "gbs": gbs,
                          "frac_hbm": gbs / bw_peak}))
    ctx.close()


if __name__ == "__main__":
    main()
