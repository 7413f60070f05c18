// encoder.cu - ViT block and encoder drivers over the operators.
//
// Reference: TransformerBlock.forward (ViTEncoder.swift:368-431; fused op
// order :433-691) and ViTEncoder.forward (ViTEncoder.swift:1235-1481): patch
// embedding, the block loop with the token-pruning step inside it
// (:1339-1396; here after `prune_after_block` blocks, all blocks global), the
// RoPE rows of the kept tokens gathered alongside their features
// (TokenPruner.swift:65-69). Per block: LN1 -> QKV GEMM (+bias, +RoPE
// epilogue) -> attention -> out-proj GEMM (+bias, +residual, in place) -> LN2
// -> fc1 GEMM (+bias, +GELU) -> fc2 GEMM (+bias, +residual, in place).
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace sam3 {
sam3_status_t ensure_workspace(sam3_ctx_t* ctx);

namespace {

__global__ void iota_kernel(int32_t* idx, int per, long long total) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < total) idx[i] = (int32_t)(i % per);
}

sam3_status_t check_block_weights(sam3_ctx_t* ctx, const sam3_block_weights_t* w) {
  if (!w) return set_error(ctx, SAM3_ERR_INVALID_ARG, "block: null weights");
  const int D = ctx->cfg.embed_dim, F = ctx->cfg.mlp_hidden;
  if (w->qkv.n != 3 * D || w->qkv.k != D || w->proj.n != D || w->proj.k != D ||
      w->fc1.n != F || w->fc1.k != D || w->fc2.n != D || w->fc2.k != F)
    return set_error(ctx, SAM3_ERR_SHAPE, "block: weight shapes do not match the config");
  return SAM3_OK;
}

// rope_pos null: rope is a table of rope_rows full rows (row r % rope_rows);
// otherwise the pair-major axial table of rope_rows coordinates with per-row
// coordinates (gemm_palette).
sam3_status_t attention_block(sam3_ctx_t* ctx, uint16_t* x, int batch, int seq,
                              const sam3_block_weights_t* w, const float* rope, int rope_rows,
                              const int32_t* rope_pos = nullptr) {
  const int D = ctx->cfg.embed_dim, H = ctx->cfg.num_heads;
  const int m = batch * seq;
  sam3_status_t st;
  if ((st = layernorm(ctx, x, m, D, w->ln1_gamma, w->ln1_beta, ctx->cfg.ln_eps, ctx->ln)) != SAM3_OK)
    return st;
  if ((st = gemm_palette(ctx, ctx->ln, m, D, w->qkv.idx, w->qkv.palette, w->qkv.bias, 3 * D,
                         SAM3_EPI_BIAS_ROPE_QKV, nullptr, rope, rope_rows, ctx->qkv,
                         rope_pos)) != SAM3_OK)
    return st;
  if ((st = attention(ctx, ctx->qkv, batch, seq, H, 64, 0.125f, ctx->attn)) != SAM3_OK) return st;
  return gemm_palette(ctx, ctx->attn, m, D, w->proj.idx, w->proj.palette, w->proj.bias, D,
                      SAM3_EPI_BIAS_RESIDUAL, x, nullptr, 1, x);
}

sam3_status_t mlp_block(sam3_ctx_t* ctx, uint16_t* x, int m, const sam3_block_weights_t* w) {
  const int D = ctx->cfg.embed_dim, F = ctx->cfg.mlp_hidden;
  sam3_status_t st;
  if ((st = layernorm(ctx, x, m, D, w->ln2_gamma, w->ln2_beta, ctx->cfg.ln_eps, ctx->ln)) != SAM3_OK)
    return st;
  if ((st = gemm_palette(ctx, ctx->ln, m, D, w->fc1.idx, w->fc1.palette, w->fc1.bias, F,
                         SAM3_EPI_BIAS_GELU, nullptr, nullptr, 1, ctx->hidden)) != SAM3_OK)
    return st;
  return gemm_palette(ctx, ctx->hidden, m, F, w->fc2.idx, w->fc2.palette, w->fc2.bias, D,
                      SAM3_EPI_BIAS_RESIDUAL, x, nullptr, 1, x);
}

sam3_status_t check_rows(sam3_ctx_t* ctx, long long rows) {
  if (rows <= 0) return set_error(ctx, SAM3_ERR_SHAPE, "block: empty input");
  if ((size_t)rows > ctx->block_rows)
    return set_error(ctx, SAM3_ERR_SHAPE, "block: %lld rows exceed the context capacity %zu "
                     "(raise max_batch)", rows, ctx->block_rows);
  return SAM3_OK;
}

// Runs the encoder on a device image; returns the final residual stream
// (pointer into the workspace) and its rows per image; writes kept indices.
sam3_status_t encoder_run(sam3_ctx_t* ctx, const void* image, bool rgba, int batch,
                          const sam3_encoder_weights_t* w, int32_t* idx, const uint16_t** out,
                          int* rows_out) {
  const sam3_encoder_config_t& c = ctx->cfg;
  if (!image || !w || !idx) return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder: null pointer");
  if (batch <= 0 || batch > c.max_batch)
    return set_error(ctx, SAM3_ERR_SHAPE, "encoder: batch %d outside [1, max_batch=%d]", batch,
                     c.max_batch);
  if (w->num_blocks != c.num_blocks || (c.num_blocks > 0 && !w->blocks) || !w->patch_w)
    return set_error(ctx, SAM3_ERR_SHAPE, "encoder: weights do not match the config");
  sam3_status_t st;
  for (int i = 0; i < c.num_blocks; ++i)
    if ((st = check_block_weights(ctx, &w->blocks[i])) != SAM3_OK) return st;
  const int grid = c.image_size / c.patch;
  const int S = grid * grid, D = c.embed_dim;
  const bool pruned = c.prune_after_block > 0 && c.prune_after_block <= c.num_blocks &&
                      c.keep_tokens < S;
  const int keep = pruned ? c.keep_tokens : S;
  if ((st = rope_setup(ctx)) != SAM3_OK) return st;
  if ((st = patch_embed(ctx, image, rgba, batch, c.image_size, c.image_size, w->patch_w,
                        w->patch_b, c.patch, D, ctx->x, ctx->cols, ctx->patch_wp)) != SAM3_OK)
    return st;
  uint16_t* cur = ctx->x;
  int rows = S;
  // the QKV epilogue rotates by the axial table and each row's coordinates
  const int32_t* rope_pos = ctx->rope_pos_grid;
  for (int blk = 0; blk <= c.num_blocks; ++blk) {
    if (pruned && blk == c.prune_after_block) {
      if ((st = prune(ctx, cur, batch, S, D, keep, c.score_norm, c.keep_order, ctx->rope, S, 64,
                      ctx->xp, ctx->rope_pruned, idx, ctx->scores)) != SAM3_OK)
        return st;
      if ((st = rope_pos_from_idx(ctx, idx, batch * keep, grid, ctx->rope_pos_pruned)) != SAM3_OK)
        return st;
      cur = ctx->xp;
      rows = keep;
      rope_pos = ctx->rope_pos_pruned;
    }
    if (blk == c.num_blocks) break;
    if ((st = attention_block(ctx, cur, batch, rows, &w->blocks[blk], ctx->rope_axial, grid,
                              rope_pos)) != SAM3_OK)
      return st;
    if ((st = mlp_block(ctx, cur, batch * rows, &w->blocks[blk])) != SAM3_OK) return st;
  }
  if (!pruned) {
    const long long total = (long long)batch * S;
    ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 4.0 * total);
    iota_kernel<<<(int)((total + 255) / 256), 256, 0, ctx->stream>>>(idx, S, total);
    if ((st = check_launch(ctx, "iota_kernel")) != SAM3_OK) return st;
  }
  *out = cur;
  *rows_out = rows;
  return SAM3_OK;
}

}  // namespace
}  // namespace sam3

using namespace sam3;

extern "C" {

sam3_status_t sam3_attention_block(sam3_ctx_t* ctx, uint16_t* x, int32_t batch, int32_t seq,
                                   const sam3_block_weights_t* w, const float* rope,
                                   int32_t rope_rows) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  sam3_status_t st = check_block_weights(ctx, w);
  if (st != SAM3_OK) return st;
  if ((st = check_rows(ctx, (long long)batch * seq)) != SAM3_OK) return st;
  if (!x || !rope) return set_error(ctx, SAM3_ERR_INVALID_ARG, "attention_block: null pointer");
  return attention_block(ctx, x, batch, seq, w, rope, rope_rows);
}

sam3_status_t sam3_mlp_block(sam3_ctx_t* ctx, uint16_t* x, int32_t m,
                             const sam3_block_weights_t* w) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  sam3_status_t st = check_block_weights(ctx, w);
  if (st != SAM3_OK) return st;
  if ((st = check_rows(ctx, m)) != SAM3_OK) return st;
  if (!x) return set_error(ctx, SAM3_ERR_INVALID_ARG, "mlp_block: null pointer");
  return mlp_block(ctx, x, m, w);
}

sam3_status_t sam3_vit_block(sam3_ctx_t* ctx, uint16_t* x, int32_t batch, int32_t seq,
                             const sam3_block_weights_t* w, const float* rope, int32_t rope_rows) {
  sam3_status_t st = sam3_attention_block(ctx, x, batch, seq, w, rope, rope_rows);
  if (st != SAM3_OK) return st;
  return mlp_block(ctx, x, batch * seq, w);
}

int32_t sam3_encoder_out_tokens(const sam3_ctx_t* ctx) {
  if (!ctx) return 0;
  const sam3_encoder_config_t& c = ctx->cfg;
  const int grid = c.image_size / c.patch;
  const int S = grid * grid;
  const bool pruned =
      c.prune_after_block > 0 && c.prune_after_block <= c.num_blocks && c.keep_tokens < S;
  return pruned ? c.keep_tokens : S;
}

sam3_status_t sam3_encoder_forward(sam3_ctx_t* ctx, const uint16_t* image, int32_t batch,
                                   const sam3_encoder_weights_t* w, uint16_t* feats,
                                   int32_t* idx) {
  SAM3_CHECK_CTX(ctx);
  if (!feats) return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder: null feats");
  cudaSetDevice(ctx->device);
  const uint16_t* out = nullptr;
  int rows = 0;
  sam3_status_t st = encoder_run(ctx, image, false, batch, w, idx, &out, &rows);
  if (st != SAM3_OK) return st;
  const size_t bytes = (size_t)batch * rows * ctx->cfg.embed_dim * 2;
  return check_cuda(ctx, cudaMemcpyAsync(feats, out, bytes, cudaMemcpyDeviceToDevice, ctx->stream),
                    "encoder feats copy");
}

sam3_status_t sam3_encoder_forward_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch,
                                        const sam3_encoder_weights_t* w, uint16_t* feats,
                                        int32_t* idx) {
  SAM3_CHECK_CTX(ctx);
  if (!feats) return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder: null feats");
  if (!rgba || !aligned16(rgba))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder: rgba must be a 16-byte aligned pointer");
  cudaSetDevice(ctx->device);
  const uint16_t* out = nullptr;
  int rows = 0;
  sam3_status_t st = encoder_run(ctx, rgba, true, batch, w, idx, &out, &rows);
  if (st != SAM3_OK) return st;
  const size_t bytes = (size_t)batch * rows * ctx->cfg.embed_dim * 2;
  return check_cuda(ctx, cudaMemcpyAsync(feats, out, bytes, cudaMemcpyDeviceToDevice, ctx->stream),
                    "encoder feats copy");
}

sam3_status_t sam3_encoder_forward_host(sam3_ctx_t* ctx, const uint16_t* host_image,
                                        int32_t batch, const sam3_encoder_weights_t* w,
                                        uint16_t* host_feats, int32_t* host_idx) {
  SAM3_CHECK_CTX(ctx);
  if (!host_image || !host_feats || !host_idx)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder_host: null pointer");
  if (batch <= 0 || batch > ctx->cfg.max_batch)
    return set_error(ctx, SAM3_ERR_SHAPE, "encoder_host: batch %d outside [1, %d]", batch,
                     ctx->cfg.max_batch);
  cudaSetDevice(ctx->device);
  const sam3_encoder_config_t& c = ctx->cfg;
  const size_t img_bytes = (size_t)batch * c.image_size * c.image_size * 3 * 2;
  sam3_status_t st = check_cuda(
      ctx, cudaMemcpyAsync(ctx->image, host_image, img_bytes, cudaMemcpyHostToDevice, ctx->stream),
      "encoder_host image upload");
  if (st != SAM3_OK) return st;
  const uint16_t* out = nullptr;
  int rows = 0;
  if ((st = encoder_run(ctx, ctx->image, false, batch, w, ctx->idx, &out, &rows)) != SAM3_OK)
    return st;
  const size_t fbytes = (size_t)batch * rows * c.embed_dim * 2;
  if ((st = check_cuda(ctx, cudaMemcpyAsync(host_feats, out, fbytes, cudaMemcpyDeviceToHost,
                                            ctx->stream),
                       "encoder_host feats download")) != SAM3_OK)
    return st;
  if ((st = check_cuda(ctx, cudaMemcpyAsync(host_idx, ctx->idx, (size_t)batch * rows * 4,
                                            cudaMemcpyDeviceToHost, ctx->stream),
                       "encoder_host idx download")) != SAM3_OK)
    return st;
  return sam3_sync(ctx);
}

sam3_status_t sam3_encoder_submit_host(sam3_ctx_t* ctx, const uint16_t* host_image,
                                       int32_t n_images, const sam3_encoder_weights_t* w,
                                       uint16_t* host_feats, int32_t* host_idx,
                                       uint64_t* ticket) {
  SAM3_CHECK_CTX(ctx);
  if (!host_image || !host_feats || !host_idx || !ticket)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder_submit_host: null pointer");
  if (n_images <= 0)
    return set_error(ctx, SAM3_ERR_SHAPE, "encoder_submit_host: n_images %d", n_images);
  cudaSetDevice(ctx->device);
  const sam3_encoder_config_t& c = ctx->cfg;
  const int B = c.max_batch;
  const int rows = sam3_encoder_out_tokens(ctx);
  const size_t img_elems = (size_t)c.image_size * c.image_size * 3;
  const size_t img_bytes = (size_t)B * img_elems * 2;
  const size_t feat_bytes = (size_t)B * rows * c.embed_dim * 2;
  const size_t idx_bytes = ((size_t)B * rows * 4 + 255) / 256 * 256;
  const size_t set_bytes = img_bytes + feat_bytes + idx_bytes;
  sam3_status_t st;
  // streams, events and pinned words, made on first use; whatever a failed
  // attempt made is kept (sam3_ctx_destroy frees it) and the rest retried
  if (!ctx->copy_stream &&
      (st = check_cuda(ctx, cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking),
                       "upload stream")) != SAM3_OK)
    return st;
  if (!ctx->down_stream &&
      (st = check_cuda(ctx, cudaStreamCreateWithFlags(&ctx->down_stream, cudaStreamNonBlocking),
                       "download stream")) != SAM3_OK)
    return st;
  if (!ctx->pipe_err &&
      (st = check_cuda(ctx, cudaHostAlloc(&ctx->pipe_err, sizeof(int) * ctx->kPipeTickets,
                                          cudaHostAllocDefault),
                       "pinned error words")) != SAM3_OK)
    return st;
  for (cudaEvent_t& e : ctx->pipe_ev)
    if (!e && (st = check_cuda(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming),
                               "pipeline event")) != SAM3_OK)
      return st;
  for (cudaEvent_t& e : ctx->pipe_done)
    if (!e && (st = check_cuda(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming),
                               "pipeline event")) != SAM3_OK)
      return st;
  const cudaStream_t up = ctx->copy_stream, down = ctx->down_stream;
  // on an error after the first copy, nothing may still be in flight against
  // the caller's host buffers when this returns
  auto drain = [&](sam3_status_t s) {
    cudaStreamSynchronize(up);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamSynchronize(down);
    return s;
  };
  if (ctx->pipe_bytes < 2 * set_bytes && (ctx->fault & SAM3_FAULT_ALLOC))
    return set_error(ctx, SAM3_ERR_OOM, "encoder_submit_host: injected allocation failure");
  if (ctx->pipe_bytes < 2 * set_bytes) {
    if (ctx->pipe_mem) {
      drain(SAM3_OK);
      cudaFree(ctx->pipe_mem);
      ctx->pipe_mem = nullptr;
      ctx->pipe_bytes = 0;
    }
    if (cudaMalloc(&ctx->pipe_mem, 2 * set_bytes) != cudaSuccess) {
      cudaGetLastError();
      return set_error(ctx, SAM3_ERR_OOM, "encoder_submit_host: %zu bytes of staging",
                       2 * set_bytes);
    }
    ctx->pipe_bytes = 2 * set_bytes;
  }
  uint16_t* img[2];
  uint16_t* feats[2];
  int32_t* idx[2];
  for (int b = 0; b < 2; ++b) {
    char* base = ctx->pipe_mem + b * set_bytes;
    img[b] = reinterpret_cast<uint16_t*>(base);
    feats[b] = reinterpret_cast<uint16_t*>(base + img_bytes);
    idx[b] = reinterpret_cast<int32_t*>(base + img_bytes + feat_bytes);
  }
  cudaEvent_t* in_done = ctx->pipe_ev;       // chunk's images are on the device
  cudaEvent_t* img_free = ctx->pipe_ev + 2;  // the encoder has finished with them
  cudaEvent_t* out_ready = ctx->pipe_ev + 4; // chunk's features are staged
  cudaEvent_t* out_done = ctx->pipe_ev + 6;  // and copied to the host
  const int chunks = (n_images + B - 1) / B;
  const uint64_t g0 = ctx->pipe_chunks;  // global number of this call's first chunk
  auto count = [&](int ch) { return std::min(B, n_images - ch * B); };
  // Three streams: uploads, the encoder (ctx->stream) and downloads. Staging
  // set g & 1 is reused by chunk g + 2, so chunk g's upload waits until the
  // encoder of chunk g - 2 has read its images, and its encoder until the
  // download of chunk g - 2 has drained its features. Nothing else orders the
  // streams, so a later call's upload runs under this call's encoder and this
  // call's download under the later call's encoder.
  auto upload = [&](int ch) -> sam3_status_t {
    const uint64_t g = g0 + ch;
    const int b = (int)(g & 1);
    if (g >= 2) cudaStreamWaitEvent(up, img_free[b], 0);
    sam3_status_t s = check_cuda(
        ctx, cudaMemcpyAsync(img[b], host_image + (size_t)ch * B * img_elems,
                             (size_t)count(ch) * img_elems * 2, cudaMemcpyHostToDevice, up),
        "image upload");
    if (s == SAM3_OK) s = check_cuda(ctx, cudaEventRecord(in_done[b], up), "event");
    return s;
  };
  if ((st = upload(0)) != SAM3_OK) return drain(st);
  for (int ch = 0; ch < chunks; ++ch) {
    const uint64_t g = g0 + ch;
    const int b = (int)(g & 1), nb = count(ch);
    if (ch + 1 < chunks && (st = upload(ch + 1)) != SAM3_OK) return drain(st);
    cudaStreamWaitEvent(ctx->stream, in_done[b], 0);
    if (g >= 2) cudaStreamWaitEvent(ctx->stream, out_done[b], 0);
    const uint16_t* out = nullptr;
    int r = 0;
    if ((st = encoder_run(ctx, img[b], false, nb, w, idx[b], &out, &r)) != SAM3_OK) return drain(st);
    const size_t fb = (size_t)nb * r * c.embed_dim * 2;
    if ((st = check_cuda(ctx, cudaEventRecord(img_free[b], ctx->stream), "event")) != SAM3_OK ||
        (st = check_cuda(ctx, cudaMemcpyAsync(feats[b], out, fb, cudaMemcpyDeviceToDevice,
                                              ctx->stream),
                         "feats staging")) != SAM3_OK ||
        (st = check_cuda(ctx, cudaEventRecord(out_ready[b], ctx->stream), "event")) != SAM3_OK)
      return drain(st);
    cudaStreamWaitEvent(down, out_ready[b], 0);
    if ((st = check_cuda(ctx, cudaMemcpyAsync(host_feats + (size_t)ch * B * r * c.embed_dim,
                                              feats[b], fb, cudaMemcpyDeviceToHost, down),
                         "feats download")) != SAM3_OK ||
        (st = check_cuda(ctx, cudaMemcpyAsync(host_idx + (size_t)ch * B * r, idx[b],
                                              (size_t)nb * r * 4, cudaMemcpyDeviceToHost, down),
                         "idx download")) != SAM3_OK ||
        (st = check_cuda(ctx, cudaEventRecord(out_done[b], down), "event")) != SAM3_OK)
      return drain(st);
  }
  ctx->pipe_chunks = g0 + chunks;
  // the device error word as the last chunk's encoder left it, then the
  // ticket's event: both behind the last download
  const uint64_t t = ++ctx->pipe_tickets;
  const int slot = (int)(t % ctx->kPipeTickets);
  if ((st = check_cuda(ctx, cudaMemcpyAsync(ctx->pipe_err + slot, ctx->dev_err, sizeof(int),
                                            cudaMemcpyDeviceToHost, down),
                       "error word download")) != SAM3_OK ||
      (st = check_cuda(ctx, cudaEventRecord(ctx->pipe_done[slot], down), "event")) != SAM3_OK)
    return drain(st);
  *ticket = t;
  return SAM3_OK;
}

sam3_status_t sam3_encoder_wait_host(sam3_ctx_t* ctx, uint64_t ticket) {
  SAM3_CHECK_CTX(ctx);
  if (ticket == 0 || ticket > ctx->pipe_tickets)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "encoder_wait_host: ticket %llu not issued",
                     (unsigned long long)ticket);
  cudaSetDevice(ctx->device);
  // The download stream runs submissions in order: a ticket older than the
  // ones still held is complete once the oldest held one is.
  const uint64_t oldest =
      ctx->pipe_tickets > (uint64_t)ctx->kPipeTickets ? ctx->pipe_tickets - ctx->kPipeTickets + 1
                                                      : 1;
  const int slot = (int)(std::max(ticket, oldest) % ctx->kPipeTickets);
  sam3_status_t st =
      check_cuda(ctx, cudaEventSynchronize(ctx->pipe_done[slot]), "encoder_wait_host");
  if (st != SAM3_OK) return st;
  return device_error_status(ctx, ctx->pipe_err[slot]);
}

sam3_status_t sam3_encoder_forward_host_pipelined(sam3_ctx_t* ctx, const uint16_t* host_image,
                                                  int32_t n_images,
                                                  const sam3_encoder_weights_t* w,
                                                  uint16_t* host_feats, int32_t* host_idx) {
  uint64_t t = 0;
  sam3_status_t st = sam3_encoder_submit_host(ctx, host_image, n_images, w, host_feats, host_idx, &t);
  if (st != SAM3_OK) return st;
  st = sam3_encoder_wait_host(ctx, t);
  const sam3_status_t s2 = sam3_sync(ctx);  // reads and clears the device error word
  return st != SAM3_OK ? st : s2;
}

}  // extern "C"
