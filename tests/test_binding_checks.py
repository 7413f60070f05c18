"""The Python binding's own argument checks (CPU only, no context on a GPU):
host buffers handed to the host-buffer encoder entry points and device
buffers handed to upload/download are checked for layout and size before any
raw pointer reaches the C ABI, which cannot see either."""
import numpy as np
import pytest

F16 = np.float16


@pytest.fixture
def fake_ctx(sam3, monkeypatch):
    # A Context object with no device context behind it: every call that gets
    # past the binding's checks reaches the library with a null handle, which
    # it rejects with SAM3_ERR_INVALID_ARG before touching any pointer.
    ctx = sam3.Context.__new__(sam3.Context)
    ctx.handle = None
    ctx.config = sam3.default_config(embed_dim=256, num_heads=4, mlp_hidden=512, num_blocks=2,
                                     image_size=112, prune_after_block=1, keep_tokens=32)
    ctx._buffers = set()
    ctx._in_flight = {}
    monkeypatch.setattr(sam3.Context, "out_tokens", property(lambda self: 32))
    return ctx


def _buf(sam3, ctx, nbytes):
    b = sam3.DeviceBuffer.__new__(sam3.DeviceBuffer)
    b.ctx, b.nbytes, b.ptr = ctx, nbytes, None
    return b


def test_upload_and_download_respect_the_device_buffer_size(sam3, fake_ctx):
    small = _buf(sam3, fake_ctx, 16)
    with pytest.raises(ValueError, match="32 bytes into a 16-byte buffer"):
        fake_ctx.upload(np.zeros(16, F16), small)
    with pytest.raises(ValueError, match="32 bytes from a 16-byte buffer"):
        fake_ctx.download(small, (16,), F16)
    with pytest.raises(sam3.SAM3Error):  # fits: reaches the library (null context)
        fake_ctx.upload(np.zeros(8, F16), small)


def _io(n=2):
    return (np.zeros((n, 112, 112, 3), F16), np.empty((n, 32, 256), F16),
            np.empty((n, 32), np.int32))


@pytest.mark.parametrize("entry", ["encoder_forward_host", "encoder_forward_host_pipelined",
                                   "encoder_submit_host"])
def test_host_entry_points_check_their_buffers(sam3, fake_ctx, entry):
    call = getattr(fake_ctx, entry)
    w = sam3.EncoderWeights()
    img, feats, idx = _io()
    with pytest.raises(sam3.SAM3Error):  # well-formed: reaches the library
        call(img, 2, w, feats, idx)
    with pytest.raises(ValueError, match="image: host array must be C-contiguous"):
        call(np.zeros((2, 112, 224, 3), F16)[:, :, ::2], 2, w, feats, idx)
    with pytest.raises(ValueError, match="image: .* bytes, needs"):
        call(img[:1], 2, w, feats, idx)
    with pytest.raises(ValueError, match="feats: element size 4, expected 2"):
        call(img, 2, w, feats.astype(np.float32), idx)
    with pytest.raises(ValueError, match="idx: .* bytes, needs"):
        call(img, 2, w, feats, idx[:, :31].copy())
    ro = feats.copy()
    ro.setflags(write=False)
    with pytest.raises(ValueError, match="feats: host array is read-only"):
        call(img, 2, w, ro, idx)


def test_wait_host_without_a_context_is_an_error(sam3, fake_ctx):
    with pytest.raises(sam3.SAM3Error):
        fake_ctx.encoder_wait_host(1)


def test_host_tensors_are_checked_too(sam3, fake_ctx):
    torch = pytest.importorskip("torch")
    w = sam3.EncoderWeights()
    img = torch.zeros((2, 112, 112, 3), dtype=torch.float16)
    feats = torch.empty((2, 32, 256), dtype=torch.float16)
    idx = torch.empty((2, 32), dtype=torch.int32)
    with pytest.raises(sam3.SAM3Error):
        fake_ctx.encoder_forward_host(img, 2, w, feats, idx)
    with pytest.raises(ValueError, match="feats: host tensor must be contiguous"):
        fake_ctx.encoder_forward_host(img, 2, w, feats.transpose(1, 2), idx)
    with pytest.raises(ValueError, match="idx: element size 8, expected 4"):
        fake_ctx.encoder_forward_host(img, 2, w, feats, idx.long())
