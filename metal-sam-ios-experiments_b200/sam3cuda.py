"""ctypes binding of libsam3cuda's C ABI (include/sam3cuda.h).

Every call goes straight to the CUDA library; there is no CPU fallback. If the
shared object is missing the import fails with an ImportError that says how to
build it. Errors come back as :class:`SAM3Error` carrying the library's status
code and message, the Python face of the reference's ``throws SAM3Error``
(SAM3MetalPipeline.swift:176-208).

Device tensors may be given as :class:`DeviceBuffer`, as any object with a
``data_ptr()`` method (e.g. a CUDA ``torch.Tensor``), or as a raw integer
device address.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsam3cuda.so")

OK, ERR_INVALID_ARG, ERR_SHAPE, ERR_OOM, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED = range(7)
EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL, EPI_BIAS_ROPE_QKV = range(4)
FAULT_NONE, FAULT_ALLOC, FAULT_LAUNCH = 0, 1, 2
SCORE_L2, SCORE_L1 = 0, 1
ORDER_INDEX, ORDER_SCORE = 0, 1

STATUS_NAMES = {0: "SAM3_OK", 1: "SAM3_ERR_INVALID_ARG", 2: "SAM3_ERR_SHAPE", 3: "SAM3_ERR_OOM",
                4: "SAM3_ERR_CUDA", 5: "SAM3_ERR_TIMEOUT", 6: "SAM3_ERR_UNSUPPORTED"}

# Every symbol the header declares: (name, restype, argtypes).
_P, _I, _F, _SZ = C.c_void_p, C.c_int32, C.c_float, C.c_size_t


class EncoderConfig(C.Structure):
    _fields_ = [("embed_dim", C.c_int32), ("num_heads", C.c_int32), ("mlp_hidden", C.c_int32),
                ("num_blocks", C.c_int32), ("patch", C.c_int32), ("image_size", C.c_int32),
                ("prune_after_block", C.c_int32), ("keep_tokens", C.c_int32),
                ("score_norm", C.c_int32), ("keep_order", C.c_int32), ("ln_eps", C.c_float),
                ("rope_theta", C.c_float), ("max_batch", C.c_int32)]


class PaletteLinear(C.Structure):
    _fields_ = [("idx", C.c_void_p), ("palette", C.c_void_p), ("bias", C.c_void_p),
                ("n", C.c_int32), ("k", C.c_int32)]


class BlockWeights(C.Structure):
    _fields_ = [("ln1_gamma", C.c_void_p), ("ln1_beta", C.c_void_p),
                ("qkv", PaletteLinear), ("proj", PaletteLinear),
                ("ln2_gamma", C.c_void_p), ("ln2_beta", C.c_void_p),
                ("fc1", PaletteLinear), ("fc2", PaletteLinear)]


class EncoderWeights(C.Structure):
    _fields_ = [("patch_w", C.c_void_p), ("patch_b", C.c_void_p),
                ("blocks", C.POINTER(BlockWeights)), ("num_blocks", C.c_int32)]


class NeckWeights(C.Structure):
    _fields_ = [("conv1_w", C.c_void_p), ("conv1_b", C.c_void_p), ("conv2_w", C.c_void_p),
                ("conv2_b", C.c_void_p), ("in_dim", C.c_int32), ("out_dim", C.c_int32)]


class WindowedEncoderWeights(C.Structure):
    _fields_ = [("patch_w", C.c_void_p), ("patch_b", C.c_void_p), ("cls_token", C.c_void_p),
                ("pos_embed", C.c_void_p), ("pos_grid", C.c_int32), ("window", C.c_int32),
                ("blocks", C.POINTER(BlockWeights)), ("num_blocks", C.c_int32)]


PROF_CLASSES = ("gemm", "attention", "layernorm", "prune", "patch", "other")


class Profile(C.Structure):
    _fields_ = [("launches", C.c_uint64 * 6), ("milliseconds", C.c_double * 6),
                ("flops", C.c_double * 6), ("bytes", C.c_double * 6)]

    def as_dict(self):
        return {name: {"launches": int(self.launches[i]), "ms": float(self.milliseconds[i]),
                       "flops": float(self.flops[i]), "bytes": float(self.bytes[i])}
                for i, name in enumerate(PROF_CLASSES)}


_S = C.c_int  # sam3_status_t
SIGNATURES = {
    "sam3_config_default": (_S, [C.POINTER(EncoderConfig)]),
    "sam3_ctx_create": (_S, [C.c_int, C.POINTER(EncoderConfig), C.POINTER(C.c_void_p)]),
    "sam3_ctx_destroy": (_S, [_P]),
    "sam3_ctx_set_stream": (_S, [_P, _P]),
    "sam3_ctx_stream": (_P, [_P]),
    "sam3_last_error": (C.c_char_p, [_P]),
    "sam3_sync": (_S, [_P]),
    "sam3_launch_count": (C.c_uint64, [_P]),
    "sam3_alloc": (_S, [_P, _SZ, C.POINTER(C.c_void_p)]),
    "sam3_free": (_S, [_P, _P]),
    "sam3_host_alloc": (_S, [_P, _SZ, C.POINTER(C.c_void_p)]),
    "sam3_host_free": (_S, [_P, _P]),
    "sam3_upload": (_S, [_P, _P, _P, _SZ]),
    "sam3_download": (_S, [_P, _P, _P, _SZ]),
    "sam3_dequant_palette": (_S, [_P, C.POINTER(PaletteLinear), _P]),
    "sam3_linear_palette": (_S, [_P, _P, _I, C.POINTER(PaletteLinear), _I, _P, _P, _I, _P]),
    "sam3_layernorm": (_S, [_P, _P, _I, _I, _P, _P, _F, _P]),
    "sam3_rope_table": (_S, [_P, _I, _I, _I, _F, _P]),
    "sam3_rope_apply": (_S, [_P, _P, _I, _I, _I, _P, _I]),
    "sam3_attention": (_S, [_P, _P, _I, _I, _I, _I, _F, _P]),
    "sam3_token_scores": (_S, [_P, _P, _I, _I, _I, _P]),
    "sam3_prune": (_S, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _I, _P, _P, _P]),
    "sam3_patch_embed": (_S, [_P, _P, _I, _I, _I, _P, _P, _I, _I, _P]),
    "sam3_patch_embed_rgba": (_S, [_P, _P, _I, _I, _I, _P, _P, _I, _I, _P]),
    "sam3_preprocess_rgba": (_S, [_P, _P, _I, _I, _I, _P]),
    "sam3_attention_block": (_S, [_P, _P, _I, _I, C.POINTER(BlockWeights), _P, _I]),
    "sam3_mlp_block": (_S, [_P, _P, _I, C.POINTER(BlockWeights)]),
    "sam3_vit_block": (_S, [_P, _P, _I, _I, C.POINTER(BlockWeights), _P, _I]),
    "sam3_encoder_forward": (_S, [_P, _P, _I, C.POINTER(EncoderWeights), _P, _P]),
    "sam3_encoder_forward_rgba": (_S, [_P, _P, _I, C.POINTER(EncoderWeights), _P, _P]),
    "sam3_restore_spatial": (_S, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "sam3_neck": (_S, [_P, _P, _I, _I, _I, C.POINTER(NeckWeights), _P]),
    "sam3_windowed_encoder_forward": (_S, [_P, _P, _I, C.POINTER(WindowedEncoderWeights), _P]),
    "sam3_windowed_encoder_forward_rgba": (_S, [_P, _P, _I, C.POINTER(WindowedEncoderWeights), _P]),
    "sam3_encoder_forward_host_pipelined": (_S, [_P, _P, _I, C.POINTER(EncoderWeights), _P, _P]),
    "sam3_encoder_forward_host": (_S, [_P, _P, _I, C.POINTER(EncoderWeights), _P, _P]),
    "sam3_encoder_submit_host": (_S, [_P, _P, _I, C.POINTER(EncoderWeights), _P, _P,
                                      C.POINTER(C.c_uint64)]),
    "sam3_encoder_wait_host": (_S, [_P, C.c_uint64]),
    "sam3_encoder_out_tokens": (C.c_int32, [_P]),
    "sam3_selftest_wait_timeout": (_S, [_P]),
    "sam3_set_fault": (_S, [_P, _I]),
    "sam3_get_fault": (C.c_int32, [_P]),
    "sam3_profile_enable": (_S, [_P, _I]),
    "sam3_profile_read": (_S, [_P, C.POINTER(Profile)]),
    "sam3_prune_noalloc": (_S, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _I, _P, _P, _P]),
}

PRUNE_NOALLOC_MAX_ROWS = 65536


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built; run `make -C {_HERE}` (or __graft_entry__.build())")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class SAM3Error(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


def ptr(x):
    """Device address of a DeviceBuffer / tensor-like / int; None stays None."""
    if x is None:
        return None
    if isinstance(x, DeviceBuffer):
        return x.ptr
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return int(x)


def default_config(**overrides) -> EncoderConfig:
    cfg = EncoderConfig()
    lib.sam3_config_default(C.byref(cfg))
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


class DeviceBuffer:
    """Device allocation owned by a Context (freed with free() or the context)."""

    def __init__(self, ctx: "Context", nbytes: int):
        self.ctx, self.nbytes = ctx, int(nbytes)
        p = C.c_void_p()
        ctx._check(lib.sam3_alloc(ctx.handle, self.nbytes, C.byref(p)))
        self.ptr = p.value
        ctx._buffers.add(self)

    def free(self):
        if self.ptr is not None:
            self.ctx._check(lib.sam3_free(self.ctx.handle, self.ptr))
            self.ctx._buffers.discard(self)
            self.ptr = None


class Context:
    """One GPU context (stream + workspace). Mirrors the per-device set-up of
    ViTEncoder.init (ViTEncoder.swift:1056-1180)."""

    def __init__(self, device: int = 0, config: EncoderConfig | None = None, **overrides):
        cfg = config if config is not None else default_config(**overrides)
        h = C.c_void_p()
        st = lib.sam3_ctx_create(device, C.byref(cfg), C.byref(h))
        if st != OK:
            raise SAM3Error(st, f"sam3_ctx_create(device={device}) failed")
        self.handle = h.value
        self.config = cfg
        self._buffers: set[DeviceBuffer] = set()
        self._in_flight: dict[int, tuple] = {}  # ticket -> host buffers of a submission

    # ---- plumbing ---------------------------------------------------------
    def _check(self, st: int):
        if st != OK:
            msg = lib.sam3_last_error(self.handle)
            raise SAM3Error(st, msg.decode() if msg else "")

    def close(self):
        if getattr(self, "handle", None):
            for b in list(self._buffers):
                b.free()
            lib.sam3_ctx_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self):
        self._check(lib.sam3_sync(self.handle))

    def set_stream(self, stream_handle):
        self._check(lib.sam3_ctx_set_stream(self.handle, stream_handle))

    @property
    def stream(self):
        return lib.sam3_ctx_stream(self.handle)

    @property
    def launches(self) -> int:
        return int(lib.sam3_launch_count(self.handle))

    def selftest_wait_timeout(self):
        """Launch the bounded-wait self-test; the next sync raises SAM3Error (TIMEOUT)."""
        self._check(lib.sam3_selftest_wait_timeout(self.handle))

    @property
    def fault(self) -> int:
        return int(lib.sam3_get_fault(self.handle))

    @fault.setter
    def fault(self, flags: int):
        self._check(lib.sam3_set_fault(self.handle, flags))

    def profile_enable(self, on: bool = True):
        self._check(lib.sam3_profile_enable(self.handle, 1 if on else 0))

    def profile_read(self) -> dict:
        p = Profile()
        self._check(lib.sam3_profile_read(self.handle, C.byref(p)))
        return p.as_dict()

    def alloc(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def upload(self, arr: np.ndarray, buf: DeviceBuffer | None = None) -> DeviceBuffer:
        arr = np.ascontiguousarray(arr)
        if buf is None:
            buf = self.alloc(arr.nbytes)
        elif isinstance(buf, DeviceBuffer) and arr.nbytes > buf.nbytes:
            raise ValueError(f"upload of {arr.nbytes} bytes into a {buf.nbytes}-byte buffer")
        self._check(lib.sam3_upload(self.handle, ptr(buf), arr.ctypes.data_as(C.c_void_p),
                                    arr.nbytes))
        return buf

    def download(self, src, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype)
        if isinstance(src, DeviceBuffer) and out.nbytes > src.nbytes:
            raise ValueError(f"download of {out.nbytes} bytes from a {src.nbytes}-byte buffer")
        self._check(lib.sam3_download(self.handle, out.ctypes.data_as(C.c_void_p), ptr(src),
                                      out.nbytes))
        return out

    # ---- operators -------------------------------------------------------------
    def dequant_palette(self, w: PaletteLinear, out):
        self._check(lib.sam3_dequant_palette(self.handle, C.byref(w), ptr(out)))

    def linear_palette(self, x, m, w: PaletteLinear, epilogue, y, residual=None, rope=None,
                       rope_rows=0):
        self._check(lib.sam3_linear_palette(self.handle, ptr(x), m, C.byref(w), epilogue,
                                            ptr(residual), ptr(rope), rope_rows, ptr(y)))

    def layernorm(self, x, m, d, gamma, beta, eps, y):
        self._check(lib.sam3_layernorm(self.handle, ptr(x), m, d, ptr(gamma), ptr(beta), eps,
                                       ptr(y)))

    def rope_table(self, grid_h, grid_w, head_dim, theta, table):
        self._check(lib.sam3_rope_table(self.handle, grid_h, grid_w, head_dim, theta, ptr(table)))

    def rope_apply(self, qkv, m, heads, head_dim, table, rope_rows):
        self._check(lib.sam3_rope_apply(self.handle, ptr(qkv), m, heads, head_dim, ptr(table),
                                        rope_rows))

    def attention(self, qkv, batch, seq, heads, head_dim, scale, o):
        self._check(lib.sam3_attention(self.handle, ptr(qkv), batch, seq, heads, head_dim, scale,
                                       ptr(o)))

    def token_scores(self, x, rows, d, norm, scores):
        self._check(lib.sam3_token_scores(self.handle, ptr(x), rows, d, norm, ptr(scores)))

    def prune(self, x, batch, seq, d, keep, norm, order, feats, idx, rope_in=None, rope_rows=0,
              rope_cols=0, rope_out=None):
        self._check(lib.sam3_prune(self.handle, ptr(x), batch, seq, d, keep, norm, order,
                                   ptr(rope_in), rope_rows, rope_cols, ptr(feats), ptr(rope_out),
                                   ptr(idx)))

    def patch_embed(self, image, batch, height, width, patch_w, patch_b, patch, dim, out):
        self._check(lib.sam3_patch_embed(self.handle, ptr(image), batch, height, width,
                                         ptr(patch_w), ptr(patch_b), patch, dim, ptr(out)))

    def attention_block(self, x, batch, seq, w: BlockWeights, rope, rope_rows):
        self._check(lib.sam3_attention_block(self.handle, ptr(x), batch, seq, C.byref(w),
                                             ptr(rope), rope_rows))

    def mlp_block(self, x, m, w: BlockWeights):
        self._check(lib.sam3_mlp_block(self.handle, ptr(x), m, C.byref(w)))

    def vit_block(self, x, batch, seq, w: BlockWeights, rope, rope_rows):
        self._check(lib.sam3_vit_block(self.handle, ptr(x), batch, seq, C.byref(w), ptr(rope),
                                       rope_rows))

    def restore_spatial(self, pruned, idx, batch, keep, seq, dim, out):
        self._check(lib.sam3_restore_spatial(self.handle, ptr(pruned), ptr(idx), batch, keep, seq,
                                             dim, ptr(out)))

    def neck(self, x, batch, height, width, w: NeckWeights, out):
        self._check(lib.sam3_neck(self.handle, ptr(x), batch, height, width, C.byref(w), ptr(out)))

    def preprocess_rgba(self, rgba, batch, height, width, rgb):
        self._check(lib.sam3_preprocess_rgba(self.handle, ptr(rgba), batch, height, width,
                                             ptr(rgb)))

    def patch_embed_rgba(self, rgba, batch, height, width, patch_w, patch_b, patch, dim, out):
        self._check(lib.sam3_patch_embed_rgba(self.handle, ptr(rgba), batch, height, width,
                                              ptr(patch_w), ptr(patch_b), patch, dim, ptr(out)))

    def encoder_forward_rgba(self, rgba, batch, w: EncoderWeights, feats, idx):
        self._check(lib.sam3_encoder_forward_rgba(self.handle, ptr(rgba), batch, C.byref(w),
                                                  ptr(feats), ptr(idx)))

    def encoder_forward(self, image, batch, w: EncoderWeights, feats, idx):
        self._check(lib.sam3_encoder_forward(self.handle, ptr(image), batch, C.byref(w),
                                             ptr(feats), ptr(idx)))

    def windowed_encoder_forward(self, image, batch, w: WindowedEncoderWeights, out):
        self._check(lib.sam3_windowed_encoder_forward(self.handle, ptr(image), batch, C.byref(w),
                                                      ptr(out)))

    def windowed_encoder_forward_rgba(self, rgba, batch, w: WindowedEncoderWeights, out):
        self._check(lib.sam3_windowed_encoder_forward_rgba(self.handle, ptr(rgba), batch,
                                                           C.byref(w), ptr(out)))

    @staticmethod
    def _host_ptr(a, nbytes, itemsize, what, write=False):
        """Address of a host buffer, after checking that an array or tensor is
        contiguous, has the element size and holds at least `nbytes`: the C ABI
        takes raw host pointers and cannot check them. A plain integer address
        is passed through (its caller vouches for its size)."""
        if isinstance(a, np.ndarray):
            if not a.flags.c_contiguous:
                raise ValueError(f"{what}: host array must be C-contiguous")
            if a.dtype.itemsize != itemsize:
                raise ValueError(f"{what}: element size {a.dtype.itemsize}, expected {itemsize}")
            if write and not a.flags.writeable:
                raise ValueError(f"{what}: host array is read-only")
            if a.nbytes < nbytes:
                raise ValueError(f"{what}: {a.nbytes} bytes, needs {nbytes}")
            return a.ctypes.data_as(C.c_void_p)
        if hasattr(a, "data_ptr") and hasattr(a, "is_contiguous"):
            if not a.is_contiguous():
                raise ValueError(f"{what}: host tensor must be contiguous")
            if a.element_size() != itemsize:
                raise ValueError(f"{what}: element size {a.element_size()}, expected {itemsize}")
            if a.numel() * a.element_size() < nbytes:
                raise ValueError(f"{what}: {a.numel() * a.element_size()} bytes, needs {nbytes}")
            return a.data_ptr()
        return ptr(a)

    def _host_io(self, n, image, feats, idx):
        side = self.config.image_size
        t = self.out_tokens
        return (self._host_ptr(image, n * side * side * 3 * 2, 2, "image"),
                self._host_ptr(feats, n * t * self.config.embed_dim * 2, 2, "feats", write=True),
                self._host_ptr(idx, n * t * 4, 4, "idx", write=True))

    def encoder_forward_host(self, image_host: np.ndarray, batch, w: EncoderWeights,
                             feats_host: np.ndarray, idx_host: np.ndarray):
        """Host buffers in and out: fp16 images [batch, H, W, 3], fp16 features
        [batch, out_tokens, D] and int32 indices [batch, out_tokens] (numpy
        arrays, contiguous tensors, or raw addresses)."""
        img, feats, idx = self._host_io(batch, image_host, feats_host, idx_host)
        self._check(lib.sam3_encoder_forward_host(self.handle, img, batch, C.byref(w), feats, idx))

    def encoder_forward_host_pipelined(self, image_host, n_images, w: EncoderWeights, feats_host,
                                       idx_host):
        """n_images from host buffers in chunks of max_batch, copies overlapped
        (buffers as for encoder_forward_host, n_images long)."""
        img, feats, idx = self._host_io(n_images, image_host, feats_host, idx_host)
        self._check(lib.sam3_encoder_forward_host_pipelined(self.handle, img, n_images,
                                                            C.byref(w), feats, idx))

    def encoder_submit_host(self, image_host, n_images, w: EncoderWeights, feats_host,
                            idx_host) -> int:
        """Enqueue n_images from host buffers (as for encoder_forward_host_pipelined)
        and return the submission's ticket at once; the buffers must stay alive
        and the outputs unread until encoder_wait_host(ticket)."""
        img, feats, idx = self._host_io(n_images, image_host, feats_host, idx_host)
        t = C.c_uint64(0)
        self._check(lib.sam3_encoder_submit_host(self.handle, img, n_images, C.byref(w), feats,
                                                 idx, C.byref(t)))
        # the buffers stay referenced until their ticket has been waited for
        self._in_flight[int(t.value)] = (image_host, feats_host, idx_host)
        return int(t.value)

    def encoder_wait_host(self, ticket: int):
        """Block until submission `ticket` (and every earlier one) is on the host."""
        self._check(lib.sam3_encoder_wait_host(self.handle, ticket))
        for t in [t for t in self._in_flight if t <= ticket]:
            del self._in_flight[t]

    @property
    def out_tokens(self) -> int:
        return int(lib.sam3_encoder_out_tokens(self.handle))


def palette_linear(idx, palette, bias, n, k) -> PaletteLinear:
    return PaletteLinear(ptr(idx), ptr(palette), ptr(bias), n, k)


def block_weights(ln1_gamma, ln1_beta, qkv, proj, ln2_gamma, ln2_beta, fc1, fc2) -> BlockWeights:
    return BlockWeights(ptr(ln1_gamma), ptr(ln1_beta), qkv, proj, ptr(ln2_gamma), ptr(ln2_beta),
                        fc1, fc2)


def neck_weights(conv1_w, conv1_b, conv2_w, conv2_b, in_dim, out_dim) -> NeckWeights:
    return NeckWeights(ptr(conv1_w), ptr(conv1_b), ptr(conv2_w), ptr(conv2_b), in_dim, out_dim)


def encoder_weights(patch_w, patch_b, blocks) -> EncoderWeights:
    arr = (BlockWeights * len(blocks))(*blocks)
    w = EncoderWeights(ptr(patch_w), ptr(patch_b), C.cast(arr, C.POINTER(BlockWeights)),
                       len(blocks))
    w._keepalive = arr  # the C struct points into this array
    return w


def windowed_encoder_weights(patch_w, patch_b, cls_token, pos_embed, pos_grid, blocks,
                             window=None) -> WindowedEncoderWeights:
    """window defaults to pos_grid, as in the reference (SAM3EncoderConfig.swift:45)."""
    arr = (BlockWeights * max(1, len(blocks)))(*blocks)
    w = WindowedEncoderWeights(ptr(patch_w), ptr(patch_b), ptr(cls_token), ptr(pos_embed),
                               pos_grid, pos_grid if window is None else window,
                               C.cast(arr, C.POINTER(BlockWeights)), len(blocks))
    w._keepalive = arr
    return w
