"""Comparison helpers shared by the tests.

Two error measures are reported. The tests gate on the normwise one,
max_rel_err, which is the spec's "max relative error" read over the whole
tensor. elem_rel_err is the elementwise relative error with an absolute
floor: |got - ref| / max(|ref|, floor). It is printed beside the normwise
figure, and gated where a test says so, so that drift on small-magnitude
outputs is visible.
"""
import numpy as np

F16 = np.float16

# Absolute floor of the elementwise relative error: outputs whose reference
# magnitude is below it are measured against it instead (fp16 activations of
# order 1; 1e-2 is a few hundred fp16 ulps of a value near 1e-2).
ELEM_FLOOR = 1e-2


def max_rel_err(got, ref):
    """Normwise max relative error: max |got - ref| / max |ref|."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / denom)


def elem_rel_err(got, ref, floor=ELEM_FLOOR):
    """Elementwise max relative error with an absolute floor:
    max over elements of |got - ref| / max(|ref|, floor)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float((np.abs(got - ref) / np.maximum(np.abs(ref), floor)).max())


def f16_ulps(got, ref):
    """Largest distance in fp16 units-in-the-last-place (same-sign values)."""
    a = np.asarray(got, F16).view(np.int16).astype(np.int64)
    b = np.asarray(ref, F16).view(np.int16).astype(np.int64)
    a = np.where(a < 0, -32768 - a, a)
    b = np.where(b < 0, -32768 - b, b)
    return int(np.abs(a - b).max())


def margin_check(got_idx, scores, keep, margin=1e-3):
    """Kept indices of one image against the oracle's scores of that image.

    The indices must agree exactly with the top-`keep` set (ties to the lower
    index) unless the keep-th / (keep+1)-th score gap is <= margin; inside
    that band only tokens whose score lies within `margin` (absolute) of the
    cut may differ. Returns the number of kept tokens that differ from the
    oracle's set."""
    scores = np.asarray(scores, np.float64)
    order = np.lexsort((np.arange(len(scores)), -scores))
    ref = np.sort(order[:keep])
    s_sorted = scores[order]
    gap = float(s_sorted[keep - 1] - s_sorted[keep]) if keep < len(scores) else np.inf
    got = np.sort(np.asarray(got_idx))
    if gap > margin:
        assert np.array_equal(got, ref), "kept set differs although the cut margin exceeds it"
        return 0
    cut = 0.5 * float(s_sorted[keep - 1] + s_sorted[keep])
    sure_in = set(np.nonzero(scores > cut + margin)[0].tolist())
    sure_out = set(np.nonzero(scores < cut - margin)[0].tolist())
    g = set(got.tolist())
    assert sure_in <= g, "a token scoring more than the margin above the cut was dropped"
    assert not (sure_out & g), "a token scoring more than the margin below the cut was kept"
    return len(g - set(ref.tolist()))


def staged_encoder(oracle, img, blocks, pw, pb, prune_after=16, keep=2592):
    """The oracle's encoder (patch embed, blocks, prune with gathered RoPE rows,
    blocks) composed from its operators, keeping the pre-prune hidden state.
    Equal bit for bit to oracle.encoder_forward (a CPU test checks that)."""
    grid = img.shape[1] // 14
    seq = grid * grid
    heads = pw.shape[0] // 64
    table = oracle.rope_table(grid, grid)
    x = oracle.patch_embed(img, pw, pb, 14)
    for blk in blocks[:prune_after]:
        x = oracle.vit_block(x, 1, seq, heads, blk, table, seq)
    pre = x
    feats, rope_rows, idx = oracle.prune(x, 1, seq, keep, rope=table)
    y = feats
    for blk in blocks[prune_after:]:
        y = oracle.vit_block(y, 1, keep, heads, blk, rope_rows, keep)
    return pre, y, idx[0]
