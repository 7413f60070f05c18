// neck.cu - the steps after the encoder: restoring the pruned tokens to their
// grid positions and the FPN-style neck (conv 1x1 then conv 3x3).
//
// Reference: TokenPruner.restoreSpatial (TokenPruner.swift:130-196), a
// scatterND of the kept rows into zeros, and NeckLayer.forward
// (ViTEncoder.swift:16-154): conv 1x1 in_dim -> out_dim + bias, then conv 3x3
// (padding 1) out_dim -> out_dim + bias, NHWC, fp16 tensors between the convs.
//
// Both convolutions run on the tcgen05 dense GEMM of gemm_palette.cu: the 1x1
// conv is the GEMM [B*H*W, in_dim] x [out_dim, in_dim]^T; the 3x3 conv is the
// GEMM of a 3x3 patch gather [rows, 9*out_dim] (tap-major, channels inner,
// zeros outside the image) with the weights reordered to the same k order,
// over row chunks that fit the context workspace.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sam3 {
namespace {

constexpr int kDevErrBadIndex = 0x201;

// One CTA per kept row: out[b, idx[b, k], :] = pruned[b, k, :]. An index
// outside [0, seq) is recorded in the device error word and skipped.
__global__ void __launch_bounds__(128) restore_scatter_kernel(const uint4* __restrict__ pruned,
                                                              const int32_t* __restrict__ idx,
                                                              int keep, int seq, int row_u4,
                                                              uint4* __restrict__ out, int* err) {
  const int k = blockIdx.x, b = blockIdx.y;
  const int s = idx[(size_t)b * keep + k];
  if (s < 0 || s >= seq) {
    if (threadIdx.x == 0) atomicExch(err, kDevErrBadIndex);
    return;
  }
  const uint4* src = pruned + ((size_t)b * keep + k) * row_u4;
  uint4* dst = out + ((size_t)b * seq + s) * row_u4;
  for (int i = threadIdx.x; i < row_u4; i += blockDim.x) dst[i] = __ldg(src + i);
}

// Rows [row0, row0 + rows) of the 3x3 patch gather of x [B, H, W, C] (NHWC):
// row r = pixel (b, y, x), column (ky*3 + kx)*C + c = x[b, y+ky-1, x+kx-1, c],
// zero outside the image. One CTA per row, 16-byte copies.
__global__ void __launch_bounds__(128) im2col3x3_kernel(const uint4* __restrict__ x, int h, int w,
                                                        int c_u4, long long row0,
                                                        uint4* __restrict__ cols) {
  const long long r = row0 + blockIdx.x;
  const int px = (int)(r % w), py = (int)((r / w) % h);
  const long long b = r / ((long long)w * h);
  uint4* dst = cols + (size_t)blockIdx.x * 9 * c_u4;
  for (int i = threadIdx.x; i < 9 * c_u4; i += blockDim.x) {
    const int tap = i / c_u4, cu = i - tap * c_u4;
    const int yy = py + tap / 3 - 1, xx = px + tap % 3 - 1;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (yy >= 0 && yy < h && xx >= 0 && xx < w) v = __ldg(x + ((b * h + yy) * w + xx) * c_u4 + cu);
    dst[i] = v;
  }
}

// OIHW [o, c, 3, 3] -> [o, (ky*3 + kx)*C + c], the gather's column order.
__global__ void reorder3x3_kernel(const __half* __restrict__ w, int cout, int cin,
                                  __half* __restrict__ wr) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)cout * 9 * cin) return;
  const int o = (int)(i / (9 * cin));
  const int rem = (int)(i - (long long)o * 9 * cin);
  const int tap = rem / cin, c = rem - tap * cin;
  wr[i] = w[((size_t)o * cin + c) * 9 + tap];
}

}  // namespace

sam3_status_t restore_spatial(sam3_ctx_t* ctx, const uint16_t* pruned, const int32_t* idx,
                              int batch, int keep, int seq, int dim, uint16_t* out) {
  if (!pruned || !idx || !out)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "restore_spatial: null pointer");
  if (batch <= 0 || keep <= 0 || seq <= 0 || dim <= 0 || keep > seq || batch > 65535)
    return set_error(ctx, SAM3_ERR_SHAPE, "restore_spatial: bad shape");
  if (dim % 8 || !aligned16(pruned) || !aligned16(out))
    return set_error(ctx, SAM3_ERR_INVALID_ARG,
                     "restore_spatial: dim %% 8 == 0 and 16-byte aligned rows required");
  const size_t out_bytes = (size_t)batch * seq * dim * 2;
  ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0,
                 (double)out_bytes + 2.0 * batch * keep * dim * 2 + 4.0 * batch * keep);
  sam3_status_t st = check_cuda(ctx, cudaMemsetAsync(out, 0, out_bytes, ctx->stream),
                                "restore_spatial zero fill");
  if (st != SAM3_OK) return st;
  restore_scatter_kernel<<<dim3(keep, batch), 128, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(pruned), idx, keep, seq, dim / 8,
      reinterpret_cast<uint4*>(out), ctx->dev_err);
  return check_launch(ctx, "restore_scatter_kernel");
}

sam3_status_t neck(sam3_ctx_t* ctx, const uint16_t* x, int batch, int h, int w,
                   const sam3_neck_weights_t* nw, uint16_t* out) {
  if (!x || !nw || !out || !nw->conv1_w || !nw->conv2_w)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "neck: null pointer");
  const int din = nw->in_dim, dout = nw->out_dim;
  if (batch <= 0 || h <= 0 || w <= 0 || din <= 0 || dout <= 0)
    return set_error(ctx, SAM3_ERR_SHAPE, "neck: empty shape");
  if (din % 64 || dout % 128)
    return set_error(ctx, SAM3_ERR_SHAPE, "neck: need in_dim %% 64 == 0 and out_dim %% 128 == 0");
  const long long rows = (long long)batch * h * w;
  const sam3_encoder_config_t& c = ctx->cfg;
  const size_t cap_mid = ctx->block_rows * (size_t)c.embed_dim;    // ln buffer, in halves
  const size_t cap_cols = ctx->block_rows * (size_t)c.mlp_hidden;  // hidden buffer, in halves
  const size_t cap_w = (size_t)c.embed_dim * ((3 * c.patch * c.patch + 63) / 64 * 64);
  if ((size_t)rows * dout > cap_mid || (size_t)9 * dout * dout > cap_w ||
      cap_cols < (size_t)9 * dout || rows > 0x7FFFFFFFll)
    return set_error(ctx, SAM3_ERR_SHAPE, "neck: shape exceeds the context workspace");
  uint16_t* mid = ctx->ln;
  uint16_t* cols = ctx->hidden;
  uint16_t* wr = ctx->patch_wp;
  // conv 1x1: [rows, din] x [dout, din]^T + b1
  sam3_status_t st = gemm_dense(ctx, x, (int)rows, din, nw->conv1_w, nw->conv1_b, dout, mid,
                                SAM3_PROF_OTHER);
  if (st != SAM3_OK) return st;
  {
    ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 4.0 * 9 * dout * dout);
    const long long nwr = 9LL * dout * dout;
    reorder3x3_kernel<<<(int)((nwr + 255) / 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const __half*>(nw->conv2_w), dout, dout, reinterpret_cast<__half*>(wr));
    if ((st = check_launch(ctx, "reorder3x3_kernel")) != SAM3_OK) return st;
  }
  // conv 3x3 over row chunks: gather, then [chunk, 9*dout] x [dout, 9*dout]^T + b2
  const long long chunk = std::min<long long>(rows, (long long)(cap_cols / (9 * (size_t)dout)));
  for (long long r0 = 0; r0 < rows; r0 += chunk) {
    const int n_rows = (int)std::min<long long>(chunk, rows - r0);
    {
      ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 2.0 * 2 * 9 * (double)n_rows * dout);
      im2col3x3_kernel<<<n_rows, 128, 0, ctx->stream>>>(reinterpret_cast<const uint4*>(mid), h, w,
                                                          dout / 8, r0,
                                                          reinterpret_cast<uint4*>(cols));
      if ((st = check_launch(ctx, "im2col3x3_kernel")) != SAM3_OK) return st;
    }
    st = gemm_dense(ctx, cols, n_rows, 9 * dout, wr, nw->conv2_b, dout, out + (size_t)r0 * dout,
                    SAM3_PROF_OTHER);
    if (st != SAM3_OK) return st;
  }
  return SAM3_OK;
}

}  // namespace sam3

using namespace sam3;

extern "C" {

sam3_status_t sam3_restore_spatial(sam3_ctx_t* ctx, const uint16_t* pruned, const int32_t* idx,
                                   int32_t batch, int32_t keep, int32_t seq, int32_t dim,
                                   uint16_t* out) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  return restore_spatial(ctx, pruned, idx, batch, keep, seq, dim, out);
}

sam3_status_t sam3_neck(sam3_ctx_t* ctx, const uint16_t* x, int32_t batch, int32_t height,
                        int32_t width, const sam3_neck_weights_t* w, uint16_t* out) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  return neck(ctx, x, batch, height, width, w, out);
}

}  // extern "C"
