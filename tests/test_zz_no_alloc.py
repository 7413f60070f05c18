"""sam3_prune_noalloc: pruning for callers that cannot allocate device memory.

Those callers (code living inside a host application that owns every device
allocation, threads that must not risk a blocking or synchronising
cudaMalloc/cudaFree, callers without a sam3 context) pass their own buffers and
the stream; the entry point keeps its per-token scores in a fixed device array
inside the library. This test calls it through the C ABI twice in a row, with
different inputs, and checks each result against sam3_prune (the context
entry point) on the same input, where the two share their kernels, so
indices, features and RoPE rows must be identical, and against the oracle's
prune, where the indices must agree wherever the score margin at the cut
exceeds 1e-3 and the gathered rows must equal the input rows they name. The
test allocates its buffers through a context; the entry point under test
allocates nothing.
"""
import ctypes as C

import numpy as np
import pytest

from util import margin_check

pytestmark = pytest.mark.gpu
F16 = np.float16


def _prune_both(ctx, sam3, x, table, batch, seq, d, keep, norm, order):
    dx = ctx.upload(x)
    drope = ctx.upload(table)
    ref_f, ref_i, ref_r = ctx.alloc(batch * keep * d * 2), ctx.alloc(batch * keep * 4), \
        ctx.alloc(batch * keep * 64 * 4)
    ctx.prune(dx, batch, seq, d, keep, norm, order, ref_f, ref_i, rope_in=drope, rope_rows=seq,
              rope_cols=64, rope_out=ref_r)
    got_f, got_i, got_r = ctx.alloc(batch * keep * d * 2), ctx.alloc(batch * keep * 4), \
        ctx.alloc(batch * keep * 64 * 4)
    st = sam3.lib.sam3_prune_noalloc(ctx.stream, dx.ptr, batch, seq, d, keep, norm, order,
                                     drope.ptr, seq, 64, got_f.ptr, got_r.ptr, got_i.ptr)
    assert st == sam3.OK
    ctx.sync()
    out = []
    for f, i, r in ((ref_f, ref_i, ref_r), (got_f, got_i, got_r)):
        out.append((ctx.download(f, (batch * keep, d), F16).view(np.uint16),
                    ctx.download(i, (batch, keep), np.int32),
                    ctx.download(r, (batch * keep, 32, 2), np.float32)))
    return out


def test_prune_noalloc_matches_context_entry_point(sam3, oracle):
    with sam3.Context(0, max_batch=2) as ctx:
        seq, d, keep = 5184, 1024, 2592
        table = oracle.rope_table(72, 72)
        # two calls in a row on different inputs: the second must not see the
        # first call's scores left in the shared scratch
        cases = [(oracle.gen_normal(61, 1, (2 * seq, d)), 2, sam3.SCORE_L2, sam3.ORDER_INDEX),
                 (oracle.gen_normal(62, 1, (1 * seq, d), 0.0, 3.0), 1, sam3.SCORE_L1,
                  sam3.ORDER_SCORE)]
        for x, batch, norm, order in cases:
            (rf, ri, rr), (gf, gi, gr) = _prune_both(ctx, sam3, x, table, batch, seq, d, keep,
                                                    norm, order)
            assert np.array_equal(gi, ri)
            assert np.array_equal(gf, rf)
            assert np.array_equal(gr, rr)
            # the oracle's prune on the same input
            of, orr, oi = oracle.prune(x, batch, seq, keep, norm=norm, order=order, rope=table)
            scores = oracle.token_scores(x, norm).astype(np.float64).reshape(batch, seq)
            for b in range(batch):
                if order == sam3.ORDER_INDEX:
                    assert (np.diff(gi[b]) > 0).all()
                margin_check(gi[b], scores[b], keep)
            rows = (gi + seq * np.arange(batch)[:, None]).reshape(-1)
            assert np.array_equal(gf, x[rows].view(np.uint16))
            assert np.array_equal(gr, table[gi.reshape(-1)])
            if np.array_equal(gi, oi):
                assert np.array_equal(gf, of.view(np.uint16)) and np.array_equal(gr, orr)


def test_prune_noalloc_rejects_sizes_beyond_its_scratch(sam3):
    # 13 images of 5184 tokens exceed the 65536-row scratch: refused up front,
    # before any pointer is touched or any kernel launched.
    assert 13 * 5184 > sam3.PRUNE_NOALLOC_MAX_ROWS
    st = sam3.lib.sam3_prune_noalloc(None, 256, 13, 5184, 1024, 2592, sam3.SCORE_L2,
                                     sam3.ORDER_INDEX, None, 0, 0, 512, None, 768)
    assert st == sam3.ERR_SHAPE
