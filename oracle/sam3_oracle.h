/*
 * sam3_oracle.h - CPU restatement of the SAM3 palettized ViT-encoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for libsam3cuda: the
 * pytest suite, the smoke check and the CPU-baseline leg of the benchmark call
 * it. Nothing in the product library links it or falls back to it.
 *
 * PARITY UNPINNED against the reference implementation itself: the reference
 * path (Swift + Metal + MPSGraph) cannot be compiled or run on this platform,
 * and its test suite holds no golden vectors for this path. The restatement is
 * instead pinned by known-answer tests derived from the reference's formulas
 * and by golden vectors from an independent float64 restatement (see
 * tests/golden/make_golden.py).
 *
 * Numerics. fp16 storage (IEEE binary16, round-to-nearest-even) at the same
 * tensor boundaries as the CUDA path, float32 arithmetic inside each operator:
 *   LN out, QKV (+bias, +RoPE on q/k), attention out, proj+bias+residual,
 *   GELU(fc1+bias), fc2+bias+residual are each rounded to fp16 once.
 * Reference files are cited per function in sam3_oracle.cpp.
 *
 * All fp16 tensors are passed as uint16_t bit patterns.
 */
#ifndef SAM3_ORACLE_H
#define SAM3_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogue selectors (same values as SAM3_EPI_* in include/sam3cuda.h). */
enum {
  SO_EPI_BIAS = 0,
  SO_EPI_BIAS_GELU = 1,
  SO_EPI_BIAS_RESIDUAL = 2,
  SO_EPI_BIAS_ROPE_QKV = 3
};
enum { SO_SCORE_L2 = 0, SO_SCORE_L1 = 1 };
enum { SO_ORDER_INDEX = 0, SO_ORDER_SCORE = 1 };

/* ---- rounding points ------------------------------------------------------ */
/* SO_ROUND_FUSED (default): the CUDA path's rounding points listed above, one
 * fp16 rounding per fused operator.
 * SO_ROUND_GRAPH: the reference's MPSGraph op boundaries, where every graph
 * op (matmul, bias add, each multiply / add of RoPE, each step of LN and
 * GELU, the residual add) returns an fp16 tensor:
 *   linear:  h(h(x w^T) + b)                 (MPSAttention.swift:113-117,
 *                                             ViTEncoder.swift:479-483)
 *   RoPE:    c = h(cos), s = h(sin); (a, b) -> (h(h(a c) - h(b s)),
 *            h(h(a s) + h(b c)))             (MPSAttention.swift:137-160;
 *                                             the cast at :151-153)
 *   residual: h(x + h(h(y w^T) + b))         (ViTEncoder.swift:559, 605)
 *   GELU:    h(h(0.5 v) * h(1 + h(erf(h(v / h(1.41421356))))))
 *                                            (ViTEncoder.swift:581-589)
 *   LN:      mean, variance (about that fp16 mean), x - mean, sqrt(var + eps),
 *            the division, * gamma, + beta each rounded to fp16
 *                                            (ViTEncoder.swift:466-474).
 * Reductions inside one op (matmul, mean, variance) accumulate in fp32 or
 * wider before their single rounding; SDPA is unchanged (fp32 inside, fp16
 * out). The mode is process-global: set it before a computation, not while
 * one runs. */
enum { SO_ROUND_FUSED = 0, SO_ROUND_GRAPH = 1 };
void so_set_rounding(int mode);
int so_rounding(void);

/* ---- seeded synthetic data (counter-based, order independent) ---------- */
/* Every value i of a tensor is a pure function of (seed, stream, i):
 * u64 = splitmix64(seed ^ mix(stream) + i * 0x9E3779B97F4A7C15). */
void so_gen_normal_f16(uint64_t seed, uint64_t stream, int64_t n, float mean,
                       float std, uint16_t* out);
void so_gen_uniform_f16(uint64_t seed, uint64_t stream, int64_t n, float lo,
                        float hi, uint16_t* out);
void so_gen_uniform_u8(uint64_t seed, uint64_t stream, int64_t n, uint8_t* out);
/* rows x 256 palette, N(0, std) rounded to fp16, sorted ascending per row. */
void so_gen_palette(uint64_t seed, uint64_t stream, int64_t rows, float std,
                    uint16_t* out);

/* ---- operators ----------------------------------------------------------- */
void so_dequant(const uint8_t* idx, const uint16_t* palette, int64_t n,
                int64_t k, uint16_t* w_out);

/* y[m,n] = epi( sum_k x[m,k] * P[n, idx[n,k]] + bias[n] ).
 * residual: fp16 [m,n] (BIAS_RESIDUAL); rope: f32 [period, head_dim/2, 2]
 * indexed by (row % rope_period) (BIAS_ROPE_QKV, n == 3*heads*head_dim). */
void so_linear(const uint16_t* x, int64_t m, const uint8_t* idx,
               const uint16_t* palette, const uint16_t* bias, int64_t n,
               int64_t k, int epilogue, const uint16_t* residual,
               const float* rope, int64_t rope_period, int heads,
               int head_dim, uint16_t* y);

/* Dense fp16 weights w[n,k] (patch embedding). */
void so_linear_dense(const uint16_t* x, int64_t m, const uint16_t* w,
                     const uint16_t* bias, int64_t n, int64_t k, uint16_t* y);

void so_layernorm(const uint16_t* x, int64_t m, int64_t d,
                  const uint16_t* gamma, const uint16_t* beta, float eps,
                  uint16_t* y);

/* table[p, j, 0..1] = (cos, sin) for token p = h*grid_w + w. */
void so_rope_table(int grid_h, int grid_w, int head_dim, float theta,
                   float* table);

/* In place on packed qkv rows [m, 3*heads*head_dim]; q and k rotated. */
void so_rope_apply(uint16_t* qkv, int64_t m, int heads, int head_dim,
                   const float* table, int64_t rope_period);

/* o[b*seq+s, h*hd+d] = softmax(q k^T * scale) v over the packed qkv rows. */
void so_attention(const uint16_t* qkv, int batch, int64_t seq, int heads,
                  int head_dim, float scale, uint16_t* o);

void so_token_scores(const uint16_t* x, int64_t rows, int64_t d, int norm,
                     float* scores);

/* Top-`keep` per image; ties -> lower index. idx is per-image token index. */
void so_select_topk(const float* scores, int batch, int64_t seq, int64_t keep,
                    int order, int32_t* idx);

void so_prune(const uint16_t* x, int batch, int64_t seq, int64_t d,
              int64_t keep, int norm, int order, const float* rope_in,
              int64_t rope_period, int rope_cols, uint16_t* feats,
              float* rope_out, int32_t* idx);

/* out [batch, seq, dim] = 0 except out[b, idx[b, k]] = pruned[b, k]. */
void so_restore_spatial(const uint16_t* pruned, const int32_t* idx, int batch, int64_t keep,
                        int64_t seq, int64_t dim, uint16_t* out);

/* Neck: x [batch, h*w, din] -> conv 1x1 (din -> dout) + b1, rounded to fp16,
 * -> conv 3x3 pad 1 (dout -> dout) + b2 -> out [batch, h, w, dout] fp16.
 * Weights OIHW: w1 [dout, din], w2 [dout, dout, 3, 3]; fp32 accumulation. */
void so_neck(const uint16_t* x, int batch, int h, int w, int din, int dout,
             const uint16_t* w1, const uint16_t* b1, const uint16_t* w2, const uint16_t* b2,
             uint16_t* out);

/* f32 RGBA [pixels, 4] in [0, 1] -> fp16 RGB [pixels, 3]: (x - mean) / std
 * per channel with the ImageNet statistics, fp32 arithmetic, IEEE division. */
void so_preprocess_rgba(const float* rgba, int64_t pixels, uint16_t* rgb);

/* NHWC fp16 image -> [b*gh*gw, dim] tokens, conv(patch x patch, stride patch)
 * with weights [dim, 3, patch, patch] and bias [dim]. */
void so_patch_embed(const uint16_t* image, int batch, int height, int width,
                    const uint16_t* w, const uint16_t* bias, int patch,
                    int dim, uint16_t* out);

typedef struct {
  const uint8_t* idx;
  const uint16_t* palette;
  const uint16_t* bias;
  int32_t n, k;
} so_palette_linear_t;

typedef struct {
  const uint16_t* ln1_gamma;
  const uint16_t* ln1_beta;
  so_palette_linear_t qkv;
  so_palette_linear_t proj;
  const uint16_t* ln2_gamma;
  const uint16_t* ln2_beta;
  so_palette_linear_t fc1;
  so_palette_linear_t fc2;
} so_block_weights_t;

/* One pre-LN block, x [batch*seq, dim] updated in place. */
void so_vit_block(uint16_t* x, int batch, int64_t seq, int dim, int heads,
                  float ln_eps, const so_block_weights_t* w, const float* rope,
                  int64_t rope_period);

/* Full encoder: patch embed, blocks, prune after `prune_after` blocks (0 =
 * never) keeping `keep` tokens. feats [batch, keep_or_seq, dim], idx
 * [batch, keep_or_seq]. */
void so_encoder_forward(const uint16_t* image, int batch, int image_size,
                        int patch, int dim, int heads, int num_blocks,
                        int prune_after, int64_t keep, int norm, int order,
                        float ln_eps, float rope_theta,
                        const uint16_t* patch_w, const uint16_t* patch_b,
                        const so_block_weights_t* blocks, uint16_t* feats,
                        int32_t* idx);

/* Checkpoint-faithful SAM3 encoder: class token (NULL: zeros) + positional
 * table [1 + pos_grid^2, dim] resized to the token grid (bilinear, half-pixel
 * centres), blocks global at i % stride == stride - 1 (stride = max(1,
 * num_blocks / 4)), windowed (window x window, class token excluded, zero
 * attention output for it) otherwise; out [batch, grid^2, dim] grid order. */
void so_windowed_encoder_forward(const uint16_t* image, int batch, int image_size, int patch,
                                 int dim, int heads, int num_blocks, int window, int pos_grid,
                                 float ln_eps, float rope_theta, const uint16_t* patch_w,
                                 const uint16_t* patch_b, const uint16_t* cls_token,
                                 const uint16_t* pos_embed, const so_block_weights_t* blocks,
                                 uint16_t* out);

/* fp16 helpers exposed for tests. */
float so_half_to_float(uint16_t h);
uint16_t so_float_to_half(float f);
int so_num_threads(void);
// Threads the OpenMP loops use from now on (n <= 0: unchanged).
void so_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
