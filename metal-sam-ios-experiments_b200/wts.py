#!/usr/bin/env python
"""SAM3WTS1 weight files with uint8-palette linears, and the offline palettizer.

The reference packs checkpoints into SAM3WTS1 files (ModelLoader.swift:60-145,
written by scripts/python_extraction/convert_npz_to_wts.py): little-endian,
magic b"SAM3WTS1", u32 entry count, then per entry u32 key length, utf-8 key,
u8 dtype (1 float16, 2 float32, 3 int32, 4 int64, 5 uint8, 255 raw), u8 rank,
u32 shape[rank], u32 byte length, payload. The reference loader ignores the
dtype and maps every payload by key.

A palettized linear weight `<key>` [n, k] is stored as two entries of that
format: `<key>` with dtype 5 (uint8 indices [n, k]) and `<key>.palette` with
dtype 1 (fp16 [n, 256], one 256-entry palette per output channel), which is
exactly what sam3_palette_linear_t points at once uploaded. Other entries are
kept as they are.

    python wts.py palettize --src model.wts --dst model_pal.wts [--iters 12]
    python wts.py info model_pal.wts

Palettizer: per output channel (row of W), a 1-D k-means with 256 centroids on
the row's K values (uniform-grid start, Lloyd iterations with nearest-centroid
assignment by midpoints); the centroids are rounded to fp16 and sorted, and
every value is then assigned to its nearest fp16 centroid, so the kernels
dequantize exactly the values the fit chose.
"""
from __future__ import annotations

import argparse
import mmap
import re
import struct
import sys

import numpy as np

MAGIC = b"SAM3WTS1"
DTYPE_CODES = {np.dtype(np.float16): 1, np.dtype(np.float32): 2, np.dtype(np.int32): 3,
               np.dtype(np.int64): 4, np.dtype(np.uint8): 5}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}
PALETTE_SUFFIX = ".palette"
PALETTE_SIZE = 256

# Linear weights of the encoder blocks: ViTEncoder's keys (ViTEncoder.swift:
# 693-721) and the checkpoint's, under the trunk prefix with mlp.fc1 / mlp.fc2
# (WeightMapper.swift:42-77).
TRUNK = "backbone.vision_backbone.trunk"
NECK = "backbone.vision_backbone.convs.3"
LINEAR_KEY = re.compile(r"^(?:backbone\.vision_backbone\.trunk\.)?blocks\.\d+\."
                        r"(attn\.qkv|attn\.proj|mlp\.lin1|mlp\.lin2|mlp\.fc1|mlp\.fc2)\.weight$")


class WtsError(ValueError):
    pass


# ------------------------------------------------------------------ format
def read_wts(path: str) -> dict:
    """key -> numpy array (read-only views of the mapped file for known
    dtypes, uint8 bytes for dtype 255), in file order."""
    with open(path, "rb") as f:
        buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    return parse_wts(memoryview(buf))


def parse_wts(buf) -> dict:
    data = memoryview(buf)
    off = 0

    def take(n):
        nonlocal off
        if n < 0 or off + n > len(data):
            raise WtsError("truncated SAM3WTS1 data")
        out = data[off:off + n]
        off += n
        return out

    if bytes(take(8)) != MAGIC:
        raise WtsError("not a SAM3WTS1 file")
    (count,) = struct.unpack("<I", take(4))
    out = {}
    for _ in range(count):
        (klen,) = struct.unpack("<I", take(4))
        if klen == 0:
            raise WtsError("empty key")
        key = bytes(take(klen)).decode("utf-8")
        code, rank = struct.unpack("<BB", take(2))
        if rank > 8:
            raise WtsError(f"{key}: rank {rank} > 8")
        shape = struct.unpack(f"<{rank}I", take(4 * rank)) if rank else ()
        (nbytes,) = struct.unpack("<I", take(4))
        payload = take(nbytes)
        dt = CODE_DTYPES.get(code)
        if dt is None:
            out[key] = np.frombuffer(payload, np.uint8)
            continue
        arr = np.frombuffer(payload, dt)
        if int(np.prod(shape, dtype=np.int64)) != arr.size:
            raise WtsError(f"{key}: shape {shape} does not match {nbytes} bytes of {dt}")
        out[key] = arr.reshape(shape)
    return out


def write_wts(path: str, entries: dict) -> None:
    """Write key -> numpy array entries (dtypes of the format's table)."""
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", len(entries)))
        for key, arr in entries.items():
            arr = np.asarray(arr)
            if not arr.flags.c_contiguous:  # (np.ascontiguousarray would turn rank 0 into 1)
                arr = arr.copy(order="C")
            code = DTYPE_CODES.get(arr.dtype)
            if code is None:
                raise WtsError(f"{key}: dtype {arr.dtype} has no SAM3WTS1 code")
            kb = key.encode("utf-8")
            f.write(struct.pack("<I", len(kb)))
            f.write(kb)
            f.write(struct.pack("<BB", code, arr.ndim))
            f.write(struct.pack(f"<{arr.ndim}I", *arr.shape))
            f.write(struct.pack("<I", arr.nbytes))
            f.write(arr.tobytes())


# ------------------------------------------------------------------ palettizer
def palettize_row(w: np.ndarray, iters: int = 12):
    """One output channel: K values -> (uint8 indices [K], fp16 palette [256])."""
    x = np.asarray(w, np.float64).ravel()
    uniq = np.unique(x.astype(np.float16).astype(np.float64))
    if uniq.size <= PALETTE_SIZE:  # representable exactly
        cent = np.concatenate([uniq, np.full(PALETTE_SIZE - uniq.size, uniq[-1])])
    else:
        xs = np.sort(x)
        # uniform grid start: Lloyd steps never raise the squared error, so the
        # fit is at least as good as uniform 8-bit quantisation of the row
        cent = np.linspace(xs[0], xs[-1], PALETTE_SIZE)
        for _ in range(iters):
            cent = np.unique(cent)
            mid = (cent[1:] + cent[:-1]) * 0.5
            lab = np.searchsorted(mid, xs)
            sums = np.bincount(lab, weights=xs, minlength=cent.size)
            cnt = np.bincount(lab, minlength=cent.size)
            keep = cnt > 0
            new = cent.copy()
            new[keep] = sums[keep] / cnt[keep]
            if np.allclose(new, cent, rtol=0, atol=1e-12):
                cent = new
                break
            cent = new
        if cent.size < PALETTE_SIZE:  # fill collapsed slots with the largest value
            cent = np.concatenate([cent, np.full(PALETTE_SIZE - cent.size, cent[-1])])
    pal = np.sort(cent.astype(np.float16))
    pf = pal.astype(np.float64)
    mid = (pf[1:] + pf[:-1]) * 0.5
    idx = np.searchsorted(mid, x).astype(np.uint8)
    return idx, pal


def palettize(w: np.ndarray, iters: int = 12):
    """W [n, k] -> (uint8 indices [n, k], fp16 palettes [n, 256])."""
    w = np.asarray(w)
    n, k = w.shape
    idx = np.empty((n, k), np.uint8)
    pal = np.empty((n, PALETTE_SIZE), np.float16)
    for r in range(n):
        idx[r], pal[r] = palettize_row(w[r], iters)
    return idx, pal


def dequantize(idx: np.ndarray, pal: np.ndarray) -> np.ndarray:
    return np.take_along_axis(pal, idx.astype(np.int64), axis=1)


def palettize_entries(entries: dict, iters: int = 12, keys=LINEAR_KEY, log=None) -> dict:
    """Entries with every matching linear weight replaced by its index entry
    and a `<key>.palette` companion; everything else unchanged."""
    out = {}
    for key, arr in entries.items():
        if keys.match(key) and arr.ndim == 2 and key + PALETTE_SUFFIX not in entries:
            idx, pal = palettize(arr, iters)
            out[key] = idx
            out[key + PALETTE_SUFFIX] = pal
            if log:
                err = np.abs(dequantize(idx, pal).astype(np.float32) - arr.astype(np.float32))
                log(f"{key} {arr.shape}: max |dW| {err.max():.3g}, mean {err.mean():.3g}")
        else:
            out[key] = arr
    return out


# ------------------------------------------------------------------ device weights
def load_encoder_weights(ctx, entries: dict, num_blocks: int, sam3):
    """Upload a palettized SAM3WTS1 dict into the context's device memory and
    return (EncoderWeights, NeckWeights or None). Keys follow the reference's
    loadWeights (ViTEncoder.swift:1204-1228 and :693-721); layer norms default
    to gamma 1, beta 0 when absent."""

    def f16(key):
        a = entries.get(key)
        if a is None:
            return None
        return ctx.upload(np.ascontiguousarray(a, np.float16))

    def linear(prefix):
        w = entries.get(prefix + ".weight")
        pal = entries.get(prefix + ".weight" + PALETTE_SUFFIX)
        if w is None or pal is None or w.dtype != np.uint8:
            raise WtsError(f"{prefix}.weight is not palettized (run `wts.py palettize`)")
        n, k = w.shape
        if pal.shape != (n, PALETTE_SIZE):
            raise WtsError(f"{prefix}.weight.palette has shape {pal.shape}, expected {(n, 256)}")
        return sam3.palette_linear(ctx.upload(np.ascontiguousarray(w)), f16(prefix + ".weight" + PALETTE_SUFFIX),
                                   f16(prefix + ".bias"), n, k)

    def ln(prefix, dim):
        g = entries.get(prefix + ".weight")
        b = entries.get(prefix + ".bias")
        g = np.ones(dim, np.float16) if g is None else g
        b = np.zeros(dim, np.float16) if b is None else b
        return ctx.upload(np.ascontiguousarray(g, np.float16)), ctx.upload(np.ascontiguousarray(b, np.float16))

    pw = entries.get("patch_embed.proj.weight")
    if pw is None:
        raise WtsError("patch_embed.proj.weight missing")
    dim = pw.shape[0]
    blocks = []
    for i in range(num_blocks):
        p = f"blocks.{i}"
        g1, b1 = ln(p + ".norm1", dim)
        g2, b2 = ln(p + ".norm2", dim)
        blocks.append(sam3.block_weights(g1, b1, linear(p + ".attn.qkv"), linear(p + ".attn.proj"), g2, b2,
                                         linear(p + ".mlp.lin1"), linear(p + ".mlp.lin2")))
    enc = sam3.encoder_weights(f16("patch_embed.proj.weight"), f16("patch_embed.proj.bias"), blocks)
    neck = None
    if "neck.0.weight" in entries and "neck.2.weight" in entries:
        w1, w2 = entries["neck.0.weight"], entries["neck.2.weight"]
        neck = sam3.neck_weights(ctx.upload(np.ascontiguousarray(w1.reshape(w1.shape[0], -1), np.float16)),
                                 f16("neck.0.bias"), f16("neck.2.weight"), f16("neck.2.bias"),
                                 w1.shape[1], w1.shape[0])
    return enc, neck


def load_windowed_encoder_weights(ctx, entries: dict, sam3, num_blocks=None, prefix=TRUNK,
                                  window=None):
    """Upload a palettized SAM3 checkpoint (the reference's keys,
    WeightMapper.swift:42-110: `<trunk>.patch_embed.proj.*`, `<trunk>.cls_token`
    (optional), `<trunk>.pos_embed` [1, 1 + g^2, dim], `<trunk>.blocks.N.norm1 /
    attn.qkv / attn.proj / norm2 / mlp.fc1 / mlp.fc2`, neck `convs.3.conv_1x1 /
    conv_3x3`) and return (WindowedEncoderWeights, NeckWeights or None).
    num_blocks defaults to the number of blocks in the file; window to the
    position grid (SAM3EncoderConfig.swift:45)."""

    def f16(key):
        a = entries.get(key)
        return None if a is None else ctx.upload(np.ascontiguousarray(a, np.float16))

    def linear(key):
        w = entries.get(key + ".weight")
        pal = entries.get(key + ".weight" + PALETTE_SUFFIX)
        if w is None or pal is None or w.dtype != np.uint8:
            raise WtsError(f"{key}.weight is not palettized (run `wts.py palettize`)")
        n, k = w.shape
        if pal.shape != (n, PALETTE_SIZE):
            raise WtsError(f"{key}.weight.palette has shape {pal.shape}, expected {(n, 256)}")
        return sam3.palette_linear(ctx.upload(np.ascontiguousarray(w)),
                                   f16(key + ".weight" + PALETTE_SUFFIX), f16(key + ".bias"), n, k)

    pw = entries.get(f"{prefix}.patch_embed.proj.weight")
    pos = entries.get(f"{prefix}.pos_embed")
    if pw is None or pos is None:
        raise WtsError(f"{prefix}.patch_embed.proj.weight / {prefix}.pos_embed missing")
    dim = pw.shape[0]
    pos = np.ascontiguousarray(pos, np.float16).reshape(-1, dim)
    pos_grid = int(round((pos.shape[0] - 1) ** 0.5))
    if pos_grid * pos_grid + 1 != pos.shape[0]:
        raise WtsError(f"{prefix}.pos_embed has {pos.shape[0]} rows, not 1 + g^2")
    if num_blocks is None:
        num_blocks = 0
        while f"{prefix}.blocks.{num_blocks}.attn.qkv.weight" in entries:
            num_blocks += 1

    def ln(key):
        g = entries.get(key + ".weight")
        b = entries.get(key + ".bias")
        g = np.ones(dim, np.float16) if g is None else g
        b = np.zeros(dim, np.float16) if b is None else b
        return (ctx.upload(np.ascontiguousarray(g, np.float16)),
                ctx.upload(np.ascontiguousarray(b, np.float16)))

    blocks = []
    for i in range(num_blocks):
        p = f"{prefix}.blocks.{i}"
        g1, b1 = ln(p + ".norm1")
        g2, b2 = ln(p + ".norm2")
        blocks.append(sam3.block_weights(g1, b1, linear(p + ".attn.qkv"), linear(p + ".attn.proj"),
                                         g2, b2, linear(p + ".mlp.fc1"), linear(p + ".mlp.fc2")))
    cls = entries.get(f"{prefix}.cls_token")
    enc = sam3.windowed_encoder_weights(
        f16(f"{prefix}.patch_embed.proj.weight"), f16(f"{prefix}.patch_embed.proj.bias"),
        None if cls is None else ctx.upload(np.ascontiguousarray(cls, np.float16).reshape(-1)),
        ctx.upload(pos), pos_grid, blocks, window=window)
    neck = None
    if f"{NECK}.conv_1x1.weight" in entries and f"{NECK}.conv_3x3.weight" in entries:
        w1 = entries[f"{NECK}.conv_1x1.weight"]
        neck = sam3.neck_weights(ctx.upload(np.ascontiguousarray(w1.reshape(w1.shape[0], -1), np.float16)),
                                 f16(f"{NECK}.conv_1x1.bias"), f16(f"{NECK}.conv_3x3.weight"),
                                 f16(f"{NECK}.conv_3x3.bias"), w1.shape[1], w1.shape[0])
    return enc, neck


# ------------------------------------------------------------------ CLI
def main(argv=None):
    ap = argparse.ArgumentParser(description="SAM3WTS1 palettized weights")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("palettize", help="replace the block linears by uint8 indices + palettes")
    p.add_argument("--src", required=True)
    p.add_argument("--dst", required=True)
    p.add_argument("--iters", type=int, default=12)
    q = sub.add_parser("info", help="list the entries of a SAM3WTS1 file")
    q.add_argument("path")
    a = ap.parse_args(argv)
    if a.cmd == "palettize":
        entries = read_wts(a.src)
        write_wts(a.dst, palettize_entries(entries, a.iters, log=lambda m: print(m, file=sys.stderr)))
        return 0
    for key, arr in read_wts(a.path).items():
        print(f"{key}\t{arr.dtype}\t{tuple(arr.shape)}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
