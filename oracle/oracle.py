"""numpy front end for the CPU oracle (oracle/libsam3oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by the CPU-baseline leg of ``bench.py``. The product library never loads
it. PARITY UNPINNED against the reference itself (its Swift/Metal path cannot
run here); pinned by known-answer tests and an independent float64
restatement (tests/golden).

fp16 tensors travel as ``np.float16`` arrays (bit-identical to uint16 views).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libsam3oracle.so")

EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL, EPI_BIAS_ROPE_QKV = 0, 1, 2, 3
SCORE_L2, SCORE_L1 = 0, 1
# Rounding points: the CUDA path's fused operators (default), or the
# reference's MPSGraph op boundaries (every graph op returns fp16).
ROUND_FUSED, ROUND_GRAPH = 0, 1
ORDER_INDEX, ORDER_SCORE = 0, 1

_lib = None


def build() -> str:
    """Compile the oracle if the shared object is missing or stale."""
    src = os.path.join(_HERE, "sam3_oracle.cpp")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class PaletteLinear(C.Structure):
    _fields_ = [("idx", C.c_void_p), ("palette", C.c_void_p), ("bias", C.c_void_p),
                ("n", C.c_int32), ("k", C.c_int32)]


class BlockWeights(C.Structure):
    _fields_ = [("ln1_gamma", C.c_void_p), ("ln1_beta", C.c_void_p),
                ("qkv", PaletteLinear), ("proj", PaletteLinear),
                ("ln2_gamma", C.c_void_p), ("ln2_beta", C.c_void_p),
                ("fc1", PaletteLinear), ("fc2", PaletteLinear)]


def _declare(L):
    P, I64, I, F, U64 = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_uint64
    sig = {
        "so_gen_normal_f16": [U64, U64, I64, F, F, P],
        "so_gen_uniform_f16": [U64, U64, I64, F, F, P],
        "so_gen_uniform_u8": [U64, U64, I64, P],
        "so_gen_palette": [U64, U64, I64, F, P],
        "so_dequant": [P, P, I64, I64, P],
        "so_linear": [P, I64, P, P, P, I64, I64, I, P, P, I64, I, I, P],
        "so_linear_dense": [P, I64, P, P, I64, I64, P],
        "so_layernorm": [P, I64, I64, P, P, F, P],
        "so_rope_table": [I, I, I, F, P],
        "so_rope_apply": [P, I64, I, I, P, I64],
        "so_attention": [P, I, I64, I, I, F, P],
        "so_token_scores": [P, I64, I64, I, P],
        "so_select_topk": [P, I, I64, I64, I, P],
        "so_prune": [P, I, I64, I64, I64, I, I, P, I64, I, P, P, P],
        "so_patch_embed": [P, I, I, I, P, P, I, I, P],
        "so_preprocess_rgba": [P, I64, P],
        "so_restore_spatial": [P, P, I, I64, I64, I64, P],
        "so_neck": [P, I, I, I, I, I, P, P, P, P, P],
        "so_vit_block": [P, I, I64, I, I, F, P, P, I64],
        "so_encoder_forward": [P, I, I, I, I, I, I, I, I64, I, I, F, F, P, P, P, P, P],
        "so_windowed_encoder_forward": [P, I, I, I, I, I, I, I, I, F, F, P, P, P, P, P, P],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = None
    L.so_set_rounding.argtypes = [C.c_int]
    L.so_set_rounding.restype = None
    L.so_rounding.restype = C.c_int
    L.so_num_threads.restype = C.c_int
    L.so_set_num_threads.argtypes = [C.c_int]
    L.so_set_num_threads.restype = None
    L.so_half_to_float.argtypes = [C.c_uint16]
    L.so_half_to_float.restype = C.c_float
    L.so_float_to_half.argtypes = [C.c_float]
    L.so_float_to_half.restype = C.c_uint16


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a


def num_threads() -> int:
    return lib().so_num_threads()


def set_num_threads(n: int) -> None:
    """OpenMP threads for the oracle's loops (process launchers such as
    torch.distributed.run set OMP_NUM_THREADS=1 per rank)."""
    lib().so_set_num_threads(int(n))


class rounding:
    """Context manager: run the oracle with the given rounding points
    (ROUND_FUSED or ROUND_GRAPH) and restore the previous mode on exit."""

    def __init__(self, mode):
        self.mode = mode

    def __enter__(self):
        self.prev = lib().so_rounding()
        lib().so_set_rounding(int(self.mode))
        return self

    def __exit__(self, *exc):
        lib().so_set_rounding(self.prev)
        return False


# ---- generators ---------------------------------------------------------------
def gen_normal(seed, stream, shape, mean=0.0, std=1.0):
    out = np.empty(shape, np.float16)
    lib().so_gen_normal_f16(seed, stream, out.size, mean, std, _p(out))
    return out


def gen_uniform(seed, stream, shape, lo=-1.0, hi=1.0):
    out = np.empty(shape, np.float16)
    lib().so_gen_uniform_f16(seed, stream, out.size, lo, hi, _p(out))
    return out


def gen_u8(seed, stream, shape):
    out = np.empty(shape, np.uint8)
    lib().so_gen_uniform_u8(seed, stream, out.size, _p(out))
    return out


def gen_palette(seed, stream, rows, std=0.02):
    out = np.empty((rows, 256), np.float16)
    lib().so_gen_palette(seed, stream, rows, std, _p(out))
    return out


# ---- operators ----------------------------------------------------------------
def dequant(idx, palette):
    idx = _c(idx, np.uint8)
    palette = _c(palette, np.float16)
    n, k = idx.shape
    out = np.empty((n, k), np.float16)
    lib().so_dequant(_p(idx), _p(palette), n, k, _p(out))
    return out


def linear(x, idx, palette, bias, epilogue=EPI_BIAS, residual=None, rope=None,
           rope_period=1, heads=16, head_dim=64):
    x = _c(x, np.float16)
    idx = _c(idx, np.uint8)
    palette = _c(palette, np.float16)
    bias = None if bias is None else _c(bias, np.float16)
    residual = None if residual is None else _c(residual, np.float16)
    rope = None if rope is None else _c(rope, np.float32)
    m, k = x.shape
    n = idx.shape[0]
    y = np.empty((m, n), np.float16)
    lib().so_linear(_p(x), m, _p(idx), _p(palette), _p(bias), n, k, epilogue,
                    _p(residual), _p(rope), rope_period, heads, head_dim, _p(y))
    return y


def linear_dense(x, w, bias):
    x = _c(x, np.float16)
    w = _c(w, np.float16)
    bias = None if bias is None else _c(bias, np.float16)
    m, k = x.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float16)
    lib().so_linear_dense(_p(x), m, _p(w), _p(bias), n, k, _p(y))
    return y


def layernorm(x, gamma=None, beta=None, eps=1e-6):
    x = _c(x, np.float16)
    m, d = x.shape
    g = None if gamma is None else _c(gamma, np.float16)
    b = None if beta is None else _c(beta, np.float16)
    y = np.empty_like(x)
    lib().so_layernorm(_p(x), m, d, _p(g), _p(b), eps, _p(y))
    return y


def rope_table(grid_h, grid_w, head_dim=64, theta=10000.0):
    t = np.empty((grid_h * grid_w, head_dim // 2, 2), np.float32)
    lib().so_rope_table(grid_h, grid_w, head_dim, theta, _p(t))
    return t


def rope_apply(qkv, heads, head_dim, table, rope_period):
    qkv = np.array(qkv, dtype=np.float16, copy=True, order="C")
    table = _c(table, np.float32)
    lib().so_rope_apply(_p(qkv), qkv.shape[0], heads, head_dim, _p(table), rope_period)
    return qkv


def attention(qkv, batch, seq, heads, head_dim, scale=None):
    qkv = _c(qkv, np.float16)
    if scale is None:
        scale = 1.0 / np.sqrt(head_dim)
    o = np.empty((batch * seq, heads * head_dim), np.float16)
    lib().so_attention(_p(qkv), batch, seq, heads, head_dim, float(scale), _p(o))
    return o


def token_scores(x, norm=SCORE_L2):
    x = _c(x, np.float16)
    s = np.empty(x.shape[0], np.float32)
    lib().so_token_scores(_p(x), x.shape[0], x.shape[1], norm, _p(s))
    return s


def select_topk(scores, batch, seq, keep, order=ORDER_INDEX):
    scores = _c(scores, np.float32)
    idx = np.empty((batch, keep), np.int32)
    lib().so_select_topk(_p(scores), batch, seq, keep, order, _p(idx))
    return idx


def prune(x, batch, seq, keep, norm=SCORE_L2, order=ORDER_INDEX, rope=None,
          rope_period=None):
    x = _c(x, np.float16)
    d = x.shape[1]
    feats = np.empty((batch * keep, d), np.float16)
    idx = np.empty((batch, keep), np.int32)
    rope_out = None
    cols = 0
    if rope is not None:
        rope = _c(rope, np.float32)
        cols = int(np.prod(rope.shape[1:]))
        rope_out = np.empty((batch * keep,) + tuple(rope.shape[1:]), np.float32)
        if rope_period is None:
            rope_period = rope.shape[0]
    lib().so_prune(_p(x), batch, seq, d, keep, norm, order, _p(rope),
                   rope_period or 1, cols, _p(feats), _p(rope_out), _p(idx))
    return feats, rope_out, idx


def preprocess_rgba(rgba):
    """f32 RGBA [..., 4] in [0, 1] -> fp16 RGB [..., 3], ImageNet-normalised
    (SAM3Predictor.swift:332-341)."""
    rgba = _c(rgba, np.float32)
    out = np.empty(rgba.shape[:-1] + (3,), np.float16)
    lib().so_preprocess_rgba(_p(rgba), rgba.size // 4, _p(out))
    return out


def restore_spatial(pruned, idx, seq):
    """pruned [B, keep, D] + idx [B, keep] -> [B, seq, D], zeros elsewhere
    (TokenPruner.swift:130-196)."""
    pruned = _c(pruned, np.float16)
    idx = _c(idx, np.int32)
    b, keep, d = pruned.shape
    out = np.empty((b, seq, d), np.float16)
    lib().so_restore_spatial(_p(pruned), _p(idx), b, keep, seq, d, _p(out))
    return out


def neck(x, batch, h, w, w1, b1, w2, b2):
    """x [B, h*w, din] -> conv1x1 + b1 -> conv3x3 (pad 1) + b2 -> [B, h, w, dout]
    (ViTEncoder.swift:54-140)."""
    x = _c(x, np.float16)
    w1, w2 = _c(w1, np.float16), _c(w2, np.float16)
    b1, b2 = _c(b1, np.float16), _c(b2, np.float16)
    dout, din = w1.shape[0], w1.shape[1]
    out = np.empty((batch, h, w, dout), np.float16)
    lib().so_neck(_p(x), batch, h, w, din, dout, _p(w1), _p(b1), _p(w2), _p(b2), _p(out))
    return out


def patch_embed(image, w, bias, patch=14):
    image = _c(image, np.float16)
    w = _c(w, np.float16)
    bias = _c(bias, np.float16)
    b, h, wd, _ = image.shape
    dim = w.shape[0]
    out = np.empty((b * (h // patch) * (wd // patch), dim), np.float16)
    lib().so_patch_embed(_p(image), b, h, wd, _p(w), _p(bias), patch, dim, _p(out))
    return out


# ---- weights ----------------------------------------------------------------------
class SyntheticBlock:
    """Seeded palettized block weights with the benchmark distributions:
    idx ~ U{0..255}, palette ~ N(0, 0.02) sorted ascending per row,
    bias ~ N(0, 0.01), LN gamma = 1, beta = 0."""

    def __init__(self, seed, layer, dim=1024, hidden=4096):
        def lin(name, n, k, tag):
            s = 1000 * layer + tag
            return {"idx": gen_u8(seed, s + 1, (n, k)),
                    "palette": gen_palette(seed, s + 2, n, 0.02),
                    "bias": gen_normal(seed, s + 3, (n,), 0.0, 0.01)}
        self.dim, self.hidden = dim, hidden
        self.ln1_gamma = np.ones(dim, np.float16)
        self.ln1_beta = np.zeros(dim, np.float16)
        self.ln2_gamma = np.ones(dim, np.float16)
        self.ln2_beta = np.zeros(dim, np.float16)
        self.qkv = lin("qkv", 3 * dim, dim, 10)
        self.proj = lin("proj", dim, dim, 20)
        self.fc1 = lin("fc1", hidden, dim, 30)
        self.fc2 = lin("fc2", dim, hidden, 40)

    def linears(self):
        return {"qkv": self.qkv, "proj": self.proj, "fc1": self.fc1, "fc2": self.fc2}

    def as_struct(self) -> BlockWeights:
        def pl(d):
            return PaletteLinear(_p(d["idx"]).value, _p(d["palette"]).value,
                                 _p(d["bias"]).value, d["idx"].shape[0], d["idx"].shape[1])
        return BlockWeights(_p(self.ln1_gamma).value, _p(self.ln1_beta).value,
                            pl(self.qkv), pl(self.proj),
                            _p(self.ln2_gamma).value, _p(self.ln2_beta).value,
                            pl(self.fc1), pl(self.fc2))


def vit_block(x, batch, seq, heads, block: SyntheticBlock, rope, rope_period,
              ln_eps=1e-6):
    x = np.array(x, dtype=np.float16, copy=True, order="C")
    rope = _c(rope, np.float32)
    w = block.as_struct()
    lib().so_vit_block(_p(x), batch, seq, x.shape[1], heads, ln_eps, C.byref(w),
                       _p(rope), rope_period)
    return x


def encoder_forward(image, blocks, patch_w, patch_b, heads=16, patch=14,
                    prune_after=16, keep=None, norm=SCORE_L2, order=ORDER_INDEX,
                    ln_eps=1e-6, theta=10000.0):
    image = _c(image, np.float16)
    b, size, _, _ = image.shape
    grid = size // patch
    seq = grid * grid
    dim = patch_w.shape[0]
    if keep is None:
        keep = seq // 2
    pruned = 0 < prune_after <= len(blocks) and keep < seq
    rows = keep if pruned else seq
    arr = (BlockWeights * len(blocks))(*[blk.as_struct() for blk in blocks])
    feats = np.empty((b, rows, dim), np.float16)
    idx = np.empty((b, rows), np.int32)
    patch_w = _c(patch_w, np.float16)
    patch_b = _c(patch_b, np.float16)
    lib().so_encoder_forward(_p(image), b, size, patch, dim, heads, len(blocks),
                             prune_after, keep, norm, order, ln_eps, theta,
                             _p(patch_w), _p(patch_b), arr, _p(feats), _p(idx))
    return feats, idx


def windowed_encoder_forward(image, blocks, patch_w, patch_b, cls_token, pos_embed, heads=16,
                             patch=14, window=None, ln_eps=1e-6, theta=10000.0):
    """Checkpoint-faithful SAM3 encoder (class token, resized positions,
    windowed/global blocks); returns [batch, grid^2, dim] in grid order.
    cls_token may be None (zeros); pos_embed [1 + pos_grid^2, dim]; window
    defaults to pos_grid, as in the reference."""
    image = _c(image, np.float16)
    b, size, _, _ = image.shape
    grid = size // patch
    dim = patch_w.shape[0]
    pos_embed = _c(pos_embed, np.float16).reshape(-1, dim)
    pos_grid = int(round((pos_embed.shape[0] - 1) ** 0.5))
    if pos_grid * pos_grid + 1 != pos_embed.shape[0]:
        raise ValueError("pos_embed must hold 1 + pos_grid^2 rows")
    window = pos_grid if window is None else window
    if grid % window:
        raise ValueError("window must divide the token grid")
    arr = (BlockWeights * max(1, len(blocks)))(*[blk.as_struct() for blk in blocks])
    out = np.empty((b, grid * grid, dim), np.float16)
    patch_w = _c(patch_w, np.float16)
    patch_b = _c(patch_b, np.float16)
    cls = None if cls_token is None else _c(cls_token, np.float16)
    lib().so_windowed_encoder_forward(_p(image), b, size, patch, dim, heads, len(blocks), window,
                                      pos_grid, ln_eps, theta, _p(patch_w), _p(patch_b), _p(cls),
                                      _p(pos_embed), arr, _p(out))
    return out
