// windowed_encoder.cu - the checkpoint-faithful SAM3 image encoder variant:
// a class token, a positional embedding bilinearly resized from its own grid,
// and windowed attention on all blocks but every (num_blocks / 4)-th.
//
// Reference: SAM3Encoder.buildGraph and buildFusedQKVAttention
// (SAM3Encoder.swift:280-366, 545-720): patch embedding, class token
// prepended (zero when the checkpoint has none), pos_embed = class position +
// pos_grid^2 positions resized to the token grid (bilinear, half-pixel
// centres), blocks with global attention at indices stride-1, 2*stride-1, ...
// (stride = max(1, num_blocks / 4)) and attention inside non-overlapping
// window x window token windows elsewhere, where the class token takes no part
// (its attention output is zero); RoPE rotates the patch tokens only; the
// output drops the class token.
//
// B200 layout: the tokens live in WINDOW-MAJOR order for the whole encoder —
// class token first, then window 0's window^2 tokens (row-major inside the
// window), window 1's, ... Every per-token operator ignores the order; a
// windowed block is attention over contiguous row groups (the grouped form of
// the attention kernel), a global block plain attention over all rows, and the
// QKV epilogue's per-row RoPE coordinates are laid out the same way once
// (no rotation for the class token). The grid order comes back in the last
// kernel.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sam3 {
namespace {

// Grid token (row-major over the grid) of window-major position p >= 1.
__device__ __forceinline__ int grid_token(int p, int grid, int window) {
  const int per = window * window, wpr = grid / window;
  const int w = (p - 1) / per, r = (p - 1) - w * per;
  const int y = r / window, x = r - y * window;
  return ((w / wpr) * window + y) * grid + (w % wpr) * window + x;
}

// Bilinear, half-pixel-centred sample of the pos_grid^2 positional table at
// grid token g, channel c; rounded to fp16 like the reference's fp16 tensor.
// Interpolation as a + f*(b - a) with IEEE fma so the oracle can match it.
__device__ __forceinline__ float upsampled_pos(const __half* __restrict__ pos, int pg, int grid,
                                               int g, int c, int dim) {
  const float ratio = __fdiv_rn((float)pg, (float)grid);
  const int gy = g / grid, gx = g - gy * grid;
  const float sy = fmaxf(__fmaf_rn((float)gy + 0.5f, ratio, -0.5f), 0.f);
  const float sx = fmaxf(__fmaf_rn((float)gx + 0.5f, ratio, -0.5f), 0.f);
  const int y0 = min((int)floorf(sy), pg - 1), x0 = min((int)floorf(sx), pg - 1);
  const int y1 = min(y0 + 1, pg - 1), x1 = min(x0 + 1, pg - 1);
  const float fy = __fsub_rn(sy, (float)y0), fx = __fsub_rn(sx, (float)x0);
  const float a = __half2float(pos[(size_t)(1 + y0 * pg + x0) * dim + c]);
  const float b = __half2float(pos[(size_t)(1 + y0 * pg + x1) * dim + c]);
  const float d = __half2float(pos[(size_t)(1 + y1 * pg + x0) * dim + c]);
  const float e = __half2float(pos[(size_t)(1 + y1 * pg + x1) * dim + c]);
  const float top = __fmaf_rn(fx, __fsub_rn(b, a), a);
  const float bot = __fmaf_rn(fx, __fsub_rn(e, d), d);
  return __half2float(__float2half_rn(__fmaf_rn(fy, __fsub_rn(bot, top), top)));
}

// x[b, p] (window-major, T = 1 + grid^2 rows per image) = class token +
// class position for p = 0, patch token + resized position otherwise.
__global__ void __launch_bounds__(128) win_embed_kernel(
    const __half* __restrict__ patches, const __half* __restrict__ cls,
    const __half* __restrict__ pos, int pg, int grid, int window, int dim,
    __half* __restrict__ x) {
  const int p = blockIdx.x, b = blockIdx.y;
  const int S = grid * grid, T = S + 1;
  __half* dst = x + ((size_t)b * T + p) * dim;
  if (p == 0) {
    for (int c = threadIdx.x; c < dim; c += blockDim.x) {
      const float v = (cls ? __half2float(cls[c]) : 0.f) + __half2float(pos[c]);
      dst[c] = __float2half_rn(v);
    }
    return;
  }
  const int g = grid_token(p, grid, window);
  const __half* src = patches + ((size_t)b * S + g) * dim;
  for (int c = threadIdx.x; c < dim; c += blockDim.x)
    dst[c] = __float2half_rn(__half2float(src[c]) + upsampled_pos(pos, pg, grid, g, c, dim));
}

// Row coordinates for the axial RoPE epilogue in window-major order:
// -1 (no rotation) for the class token, x | y << 16 of the grid token otherwise.
__global__ void win_rope_pos_kernel(int32_t* __restrict__ pos, int rows, int grid, int window) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int T = grid * grid + 1, p = r % T;
  if (p == 0) {
    pos[r] = -1;
    return;
  }
  const int g = grid_token(p, grid, window);
  pos[r] = (g % grid) | ((g / grid) << 16);
}

// out[b, g] (grid order, no class token) = x[b, p(g)].
__global__ void __launch_bounds__(128) win_unpermute_kernel(const uint4* __restrict__ x, int grid,
                                                            int window, int row_u4,
                                                            uint4* __restrict__ out) {
  const int g = blockIdx.x, b = blockIdx.y;
  const int S = grid * grid, wpr = grid / window;
  const int gy = g / grid, gx = g - gy * grid;
  const int p = 1 + ((gy / window) * wpr + gx / window) * window * window +
                (gy % window) * window + gx % window;
  const uint4* src = x + ((size_t)b * (S + 1) + p) * row_u4;
  uint4* dst = out + ((size_t)b * S + g) * row_u4;
  for (int i = threadIdx.x; i < row_u4; i += blockDim.x) dst[i] = src[i];
}

sam3_status_t check_windowed_weights(sam3_ctx_t* ctx, const sam3_windowed_encoder_weights_t* w) {
  const sam3_encoder_config_t& c = ctx->cfg;
  if (!w || !w->patch_w || !w->pos_embed || (w->num_blocks > 0 && !w->blocks))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "windowed encoder: null weights");
  const int grid = c.image_size / c.patch;
  if (w->window <= 0 || grid % w->window || w->pos_grid <= 0 || w->num_blocks < 0)
    return set_error(ctx, SAM3_ERR_SHAPE,
                     "windowed encoder: window %d must divide the %d-token grid, pos_grid > 0",
                     w->window, grid);
  const int D = c.embed_dim, F = c.mlp_hidden;
  for (int i = 0; i < w->num_blocks; ++i) {
    const sam3_block_weights_t& b = w->blocks[i];
    if (b.qkv.n != 3 * D || b.qkv.k != D || b.proj.n != D || b.proj.k != D || b.fc1.n != F ||
        b.fc1.k != D || b.fc2.n != D || b.fc2.k != F)
      return set_error(ctx, SAM3_ERR_SHAPE, "windowed encoder: block %d shapes do not match", i);
  }
  return SAM3_OK;
}

}  // namespace

// image: fp16 RGB NHWC, or f32 RGBA NHWC in [0, 1] normalised in the patch
// gather (rgba = true).
sam3_status_t windowed_encoder_run(sam3_ctx_t* ctx, const void* image, bool rgba, int batch,
                                   const sam3_windowed_encoder_weights_t* w, uint16_t* out) {
  const sam3_encoder_config_t& c = ctx->cfg;
  if (!image || !out) return set_error(ctx, SAM3_ERR_INVALID_ARG, "windowed encoder: null pointer");
  if (batch <= 0 || batch > c.max_batch)
    return set_error(ctx, SAM3_ERR_SHAPE, "windowed encoder: batch %d outside [1, max_batch=%d]",
                     batch, c.max_batch);
  sam3_status_t st = check_windowed_weights(ctx, w);
  if (st != SAM3_OK) return st;
  const int grid = c.image_size / c.patch, S = grid * grid, T = S + 1;
  const int D = c.embed_dim, H = c.num_heads, F = c.mlp_hidden;
  const int hd = D / H, win = w->window, per = win * win, nwin = S / per;
  const int rows = batch * T;
  if ((size_t)rows > ctx->token_rows)
    return set_error(ctx, SAM3_ERR_SHAPE, "windowed encoder: %d rows exceed the workspace", rows);
  if ((st = rope_setup(ctx)) != SAM3_OK) return st;
  if (ctx->rope_win_key != win) {
    const int prow = c.max_batch * T;
    win_rope_pos_kernel<<<(prow + 255) / 256, 256, 0, ctx->stream>>>(ctx->rope_pos_win, prow, grid,
                                                                     win);
    if ((st = check_launch(ctx, "win_rope_pos_kernel")) != SAM3_OK) return st;
    ctx->rope_win_key = win;
  }
  // patch tokens (grid order) into the attention scratch, then the
  // window-major residual stream with the class token and positions
  if ((st = patch_embed(ctx, image, rgba, batch, c.image_size, c.image_size, w->patch_w,
                        w->patch_b, c.patch, D, ctx->attn, ctx->cols, ctx->patch_wp)) != SAM3_OK)
    return st;
  {
    ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 2.0 * 2 * (double)rows * D);
    win_embed_kernel<<<dim3(T, batch), 128, 0, ctx->stream>>>(
        reinterpret_cast<const __half*>(ctx->attn), reinterpret_cast<const __half*>(w->cls_token),
        reinterpret_cast<const __half*>(w->pos_embed), w->pos_grid, grid, win, D,
        reinterpret_cast<__half*>(ctx->x));
    if ((st = check_launch(ctx, "win_embed_kernel")) != SAM3_OK) return st;
  }
  uint16_t* x = ctx->x;
  const int stride = std::max(1, w->num_blocks / 4);
  for (int blk = 0; blk < w->num_blocks; ++blk) {
    const sam3_block_weights_t* bw = &w->blocks[blk];
    const bool global = blk % stride == stride - 1;
    if ((st = layernorm(ctx, x, rows, D, bw->ln1_gamma, bw->ln1_beta, c.ln_eps, ctx->ln)) != SAM3_OK)
      return st;
    if ((st = gemm_palette(ctx, ctx->ln, rows, D, bw->qkv.idx, bw->qkv.palette, bw->qkv.bias,
                           3 * D, SAM3_EPI_BIAS_ROPE_QKV, nullptr, ctx->rope_axial, grid,
                           ctx->qkv, ctx->rope_pos_win)) != SAM3_OK)
      return st;
    if (global) {
      st = attention_grouped(ctx, ctx->qkv, batch, 1, T, T, 0, H, hd, 0.125f, ctx->attn);
    } else {
      st = attention_grouped(ctx, ctx->qkv, batch, nwin, per, T, 1, H, hd, 0.125f, ctx->attn);
      // the class token takes no part in windowed attention: zero output
      if (st == SAM3_OK)
        st = check_cuda(ctx, cudaMemset2DAsync(ctx->attn, (size_t)T * D * 2, 0, (size_t)D * 2,
                                               batch, ctx->stream),
                        "class-token rows");
    }
    if (st != SAM3_OK) return st;
    if ((st = gemm_palette(ctx, ctx->attn, rows, D, bw->proj.idx, bw->proj.palette, bw->proj.bias,
                           D, SAM3_EPI_BIAS_RESIDUAL, x, nullptr, 1, x)) != SAM3_OK)
      return st;
    if ((st = layernorm(ctx, x, rows, D, bw->ln2_gamma, bw->ln2_beta, c.ln_eps, ctx->ln)) != SAM3_OK)
      return st;
    if ((st = gemm_palette(ctx, ctx->ln, rows, D, bw->fc1.idx, bw->fc1.palette, bw->fc1.bias, F,
                           SAM3_EPI_BIAS_GELU, nullptr, nullptr, 1, ctx->hidden)) != SAM3_OK)
      return st;
    if ((st = gemm_palette(ctx, ctx->hidden, rows, F, bw->fc2.idx, bw->fc2.palette, bw->fc2.bias,
                           D, SAM3_EPI_BIAS_RESIDUAL, x, nullptr, 1, x)) != SAM3_OK)
      return st;
  }
  ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 2.0 * 2 * (double)batch * S * D);
  win_unpermute_kernel<<<dim3(S, batch), 128, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(x), grid, win, D / 8, reinterpret_cast<uint4*>(out));
  return check_launch(ctx, "win_unpermute_kernel");
}

}  // namespace sam3

using namespace sam3;

extern "C" sam3_status_t sam3_windowed_encoder_forward(sam3_ctx_t* ctx, const uint16_t* image,
                                                       int32_t batch,
                                                       const sam3_windowed_encoder_weights_t* w,
                                                       uint16_t* out) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  if (!aligned16(out)) return set_error(ctx, SAM3_ERR_INVALID_ARG, "windowed encoder: out must be 16-byte aligned");
  return windowed_encoder_run(ctx, image, false, batch, w, out);
}

extern "C" sam3_status_t sam3_windowed_encoder_forward_rgba(
    sam3_ctx_t* ctx, const float* rgba, int32_t batch, const sam3_windowed_encoder_weights_t* w,
    uint16_t* out) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  if (!aligned16(out) || !rgba || !aligned16(rgba))
    return set_error(ctx, SAM3_ERR_INVALID_ARG,
                     "windowed encoder: rgba and out must be 16-byte aligned pointers");
  return windowed_encoder_run(ctx, rgba, true, batch, w, out);
}
