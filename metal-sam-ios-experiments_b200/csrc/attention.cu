// attention.cu - entry point of global softmax attention over packed QKV rows.
//
// o[b*S + i, h*64 + :] = softmax_j(q_i . k_j * scale) v_j, per image b and
// head h, reading q | k | v straight from the QKV GEMM output
// [B*S, 3*H*64] (no transpose pass) and writing the [B*S, H*64] layout the
// out-projection GEMM consumes. The kernels are in attention_pp.cu (global
// attention) and attention_tc.cu (windowed attention).
//
// Reference: scaledDotProductAttention in MPSAttentionLayer
// (MPSAttention.swift:165-176, scale 1/sqrt(64), no mask) and the explicit
// QK^T -> softmax -> PV form of AttentionKernels.swift:48-68.
#include "common.cuh"
#include "internal.h"

namespace sam3 {

sam3_status_t attention_tc(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                           float scale, uint16_t* o, int groups, int img_rows, int first_row);
sam3_status_t attention_pp(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                           float scale, uint16_t* o, int groups, int img_rows, int first_row);

sam3_status_t attention_grouped(sam3_ctx_t* ctx, const uint16_t* qkv, int images, int groups,
                                int seq, int img_rows, int first_row, int heads, int head_dim,
                                float scale, uint16_t* o) {
  constexpr int kHeadDim = 64;
  if (!qkv || !o) return set_error(ctx, SAM3_ERR_INVALID_ARG, "attention: null pointer");
  if (head_dim != kHeadDim)
    return set_error(ctx, SAM3_ERR_SHAPE, "attention: head_dim must be 64 (got %d)", head_dim);
  if (images <= 0 || groups <= 0 || seq <= 0 || heads <= 0 || heads > 65535 ||
      (long long)images * groups > 65535 || first_row < 0 ||
      (long long)first_row + (long long)groups * seq > img_rows)
    return set_error(ctx, SAM3_ERR_SHAPE, "attention: bad shape");
  if (!aligned16(qkv) || !aligned16(o))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "attention: pointers must be 16-byte aligned");
  ProfScope prof(ctx, SAM3_PROF_ATTENTION,
                 4.0 * images * groups * heads * (double)seq * seq * kHeadDim,
                 8.0 * images * groups * seq * heads * kHeadDim);
  // Global attention over whole images takes the 128-key, two-query-tile
  // kernel; windows (groups of a few hundred rows) keep the 64-key kernel,
  // whose 128-row CTAs waste less on a short ragged group.
  if (groups == 1)
    return attention_pp(ctx, qkv, images, seq, heads, scale, o, groups, img_rows, first_row);
  return attention_tc(ctx, qkv, images, seq, heads, scale, o, groups, img_rows, first_row);
}

sam3_status_t attention(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                        int head_dim, float scale, uint16_t* o) {
  return attention_grouped(ctx, qkv, batch, 1, seq, seq, 0, heads, head_dim, scale, o);
}

}  // namespace sam3

using namespace sam3;

extern "C" sam3_status_t sam3_attention(sam3_ctx_t* ctx, const uint16_t* qkv, int32_t batch,
                                        int32_t seq, int32_t heads, int32_t head_dim, float scale,
                                        uint16_t* o) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  return attention(ctx, qkv, batch, seq, heads, head_dim, scale, o);
}
