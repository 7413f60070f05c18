"""SAM3WTS1 files and the per-channel palettizer (host code; no GPU).

The format is the reference's (ModelLoader.swift:60-145,
convert_npz_to_wts.py): the tests build files byte by byte from that
description and check that wts.py reads them and writes the same bytes.
"""
import struct

import numpy as np
import pytest

import wts


def _entry(key, code, shape, payload):
    kb = key.encode()
    return (struct.pack("<I", len(kb)) + kb + struct.pack("<BB", code, len(shape)) +
            struct.pack(f"<{len(shape)}I", *shape) + struct.pack("<I", len(payload)) + payload)


def _reference_bytes():
    a = np.arange(6, dtype=np.float16).reshape(2, 3)
    b = np.array([1, 2, 250, 7], np.uint8)
    c = np.array(3.5, np.float32)
    body = (_entry("blocks.0.attn.qkv.bias", 1, a.shape, a.tobytes()) +
            _entry("idx", 5, b.shape, b.tobytes()) + _entry("scale", 2, (), c.tobytes()))
    return b"SAM3WTS1" + struct.pack("<I", 3) + body, (a, b, c)


def test_reads_reference_layout_and_writes_identical_bytes(tmp_path):
    raw, (a, b, c) = _reference_bytes()
    got = wts.parse_wts(raw)
    assert list(got) == ["blocks.0.attn.qkv.bias", "idx", "scale"]
    assert np.array_equal(got["blocks.0.attn.qkv.bias"], a) and got["idx"].dtype == np.uint8
    assert np.array_equal(got["idx"], b) and float(got["scale"]) == 3.5
    p = tmp_path / "m.wts"
    wts.write_wts(str(p), {"blocks.0.attn.qkv.bias": a, "idx": b, "scale": c})
    assert p.read_bytes() == raw
    back = wts.read_wts(str(p))
    assert np.array_equal(back["idx"], b)


@pytest.mark.parametrize("bad", [b"SAM3WTS0" + b"\0" * 4, b"SAM3WTS1" + struct.pack("<I", 1)
                                 + struct.pack("<I", 4) + b"ab"])
def test_rejects_bad_magic_and_truncation(bad):
    with pytest.raises(wts.WtsError):
        wts.parse_wts(bad)


def test_palettize_exact_when_row_has_few_values():
    rng = np.random.default_rng(0)
    levels = np.sort(rng.standard_normal(200)).astype(np.float16)
    row = rng.choice(levels, 1024)
    idx, pal = wts.palettize_row(row)
    assert idx.dtype == np.uint8 and pal.dtype == np.float16 and pal.shape == (256,)
    assert np.array_equal(pal[idx].view(np.uint16), row.view(np.uint16))


def test_palettize_error_and_nearest_assignment():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((6, 1024)) * 0.02).astype(np.float32)
    idx, pal = wts.palettize(w)
    deq = wts.dequantize(idx, pal).astype(np.float64)
    # 256 levels over ~6 sigma: rms error under 1% of sigma
    rms = np.sqrt(np.mean((deq - w) ** 2))
    lo, hi = w.min(axis=1, keepdims=True), w.max(axis=1, keepdims=True)
    uni = lo + np.round((w - lo) / (hi - lo) * 255) * (hi - lo) / 255
    assert rms <= np.sqrt(np.mean((uni - w) ** 2))  # no worse than uniform 8-bit
    assert rms < 0.01 * 0.02
    assert np.all(np.diff(pal.astype(np.float32), axis=1) >= 0)
    # every value sits on (one of) its nearest palette entries
    pf = pal.astype(np.float64)
    d_all = np.abs(w[:, :, None] - pf[:, None, :]).min(axis=2)
    assert np.allclose(np.abs(deq - w), d_all, rtol=0, atol=1e-12)


def test_palettize_entries_replaces_block_linears_only(tmp_path):
    rng = np.random.default_rng(2)
    src = {"patch_embed.proj.weight": rng.standard_normal((8, 3, 2, 2)).astype(np.float16),
           "blocks.0.attn.qkv.weight": rng.standard_normal((12, 64)).astype(np.float16),
           "blocks.0.attn.qkv.bias": rng.standard_normal(12).astype(np.float16),
           "blocks.0.mlp.lin2.weight": rng.standard_normal((4, 32)).astype(np.float16)}
    out = wts.palettize_entries(src)
    assert out["patch_embed.proj.weight"] is src["patch_embed.proj.weight"]
    assert out["blocks.0.attn.qkv.weight"].dtype == np.uint8
    assert out["blocks.0.attn.qkv.weight.palette"].shape == (12, 256)
    assert out["blocks.0.mlp.lin2.weight.palette"].dtype == np.float16
    p, q = tmp_path / "a.wts", tmp_path / "b.wts"
    wts.write_wts(str(p), src)
    assert wts.main(["palettize", "--src", str(p), "--dst", str(q), "--iters", "4"]) == 0
    back = wts.read_wts(str(q))
    assert set(back) == set(out)
    assert np.array_equal(back["blocks.0.attn.qkv.weight"], out["blocks.0.attn.qkv.weight"])


def test_palettize_entries_matches_checkpoint_keys():
    # the checkpoint's trunk prefix and mlp.fc1 / mlp.fc2 names
    # (WeightMapper.swift:42-77); other modules' blocks stay dense
    rng = np.random.default_rng(3)
    t = wts.TRUNK
    src = {f"{t}.blocks.3.mlp.fc1.weight": rng.standard_normal((8, 16)).astype(np.float16),
           f"{t}.blocks.3.mlp.fc2.weight": rng.standard_normal((16, 8)).astype(np.float16),
           f"{t}.blocks.3.attn.proj.weight": rng.standard_normal((16, 16)).astype(np.float16),
           f"{t}.pos_embed": rng.standard_normal((1, 5, 16)).astype(np.float16),
           "geometry_encoder.blocks.0.attn.qkv.weight": rng.standard_normal((6, 16)).astype(np.float16)}
    out = wts.palettize_entries(src, iters=2)
    for k in ("mlp.fc1", "mlp.fc2", "attn.proj"):
        assert out[f"{t}.blocks.3.{k}.weight"].dtype == np.uint8
        assert f"{t}.blocks.3.{k}.weight.palette" in out
    assert out[f"{t}.pos_embed"] is src[f"{t}.pos_embed"]
    assert out["geometry_encoder.blocks.0.attn.qkv.weight"].dtype == np.float16
