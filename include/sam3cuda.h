/*
 * sam3cuda.h - C ABI of libsam3cuda: the SAM3 image-encoder hot path on
 * NVIDIA B200 (sm_100a).
 *
 * The path: uint8-palette (256-entry LUT per output channel) weights expanded
 * on chip into fp16 tensor-core GEMMs (QKV, attention out-projection, MLP
 * fc1/fc2) with fused epilogues (bias, 2D axial RoPE, exact GELU, residual),
 * global softmax attention, LayerNorm, patch embedding and the L2/L1 token
 * pruning top-k + gather.
 *
 * Conventions
 *  - Every entry point returns sam3_status_t; nothing aborts or throws.
 *    A failing call leaves a message readable with sam3_last_error(ctx).
 *  - fp16 tensors are IEEE binary16 passed as uint16_t (Swift: Float16 /
 *    UInt16). Tensors are row-major; token rows are [batch*seq, dim].
 *  - Device pointers are caller-owned (sam3_alloc or any CUDA allocation on the
 *    context's device). Operators are asynchronous on the context's stream;
 *    sam3_sync() waits and reports device-side errors.
 *  - One context per (host thread, GPU). Calls on one context must be
 *    serialised by the caller; different contexts are independent.
 *
 * Reference interfaces (paths relative to OrdoSAM3Sensor/Sources/Sam3Sensor/)
 * are cited beside each entry point it replaces.
 */
#ifndef SAM3CUDA_H
#define SAM3CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SAM3_OK = 0,
  SAM3_ERR_INVALID_ARG = 1, /* null pointer, bad enum, misaligned pointer  */
  SAM3_ERR_SHAPE = 2,       /* shape unsupported or inconsistent          */
  SAM3_ERR_OOM = 3,         /* device or pinned-host allocation failed     */
  SAM3_ERR_CUDA = 4,        /* CUDA runtime/driver error                   */
  SAM3_ERR_TIMEOUT = 5,     /* a kernel's bounded wait expired             */
  SAM3_ERR_UNSUPPORTED = 6  /* device is not sm_100 or feature missing     */
} sam3_status_t;

/* Epilogue selectors of sam3_linear_palette. */
typedef enum {
  SAM3_EPI_BIAS = 0,          /* y = acc + b                                 */
  SAM3_EPI_BIAS_GELU = 1,     /* y = gelu_erf(acc + b)                       */
  SAM3_EPI_BIAS_RESIDUAL = 2, /* y = residual + acc + b (y may == residual)  */
  SAM3_EPI_BIAS_ROPE_QKV = 3  /* y = rope(acc + b) on the q and k thirds     */
} sam3_epilogue_t;

typedef enum { SAM3_SCORE_L2 = 0, SAM3_SCORE_L1 = 1 } sam3_score_norm_t;
typedef enum { SAM3_ORDER_INDEX = 0, SAM3_ORDER_SCORE = 1 } sam3_keep_order_t;

typedef struct sam3_ctx sam3_ctx_t;

/* Encoder configuration. Reference: SAM3EncoderConfig.swift:6-64 and the
 * WeightMapper.swift:23-38 constants; the defaults follow the benchmark spec
 * (all-global 32 blocks, prune to 50% after block 16 by L2 norm, index order). */
typedef struct {
  int32_t embed_dim;         /* 1024 */
  int32_t num_heads;         /* 16 (head_dim must be 64) */
  int32_t mlp_hidden;        /* 4096 */
  int32_t num_blocks;        /* 32 */
  int32_t patch;             /* 14 */
  int32_t image_size;        /* 1008 (square) */
  int32_t prune_after_block; /* 16; 0 disables pruning */
  int32_t keep_tokens;       /* 2592 */
  int32_t score_norm;        /* sam3_score_norm_t */
  int32_t keep_order;        /* sam3_keep_order_t */
  float ln_eps;              /* 1e-6 */
  float rope_theta;          /* 10000 */
  int32_t max_batch;         /* images per sam3_encoder_forward call */
} sam3_encoder_config_t;

/* One palettized linear layer, device pointers: idx uint8 [n, k] (row-major,
 * PyTorch [out, in]), palette fp16 [n, 256], bias fp16 [n] (may be NULL).
 * W[r, c] = palette[r, idx[r, c]]; Y = X * W^T + b. */
typedef struct {
  const uint8_t* idx;
  const uint16_t* palette;
  const uint16_t* bias;
  int32_t n, k;
} sam3_palette_linear_t;

/* Weights of one pre-LN ViT block (device pointers). Reference:
 * TransformerBlock.loadWeights, ViTEncoder.swift:693-721. */
typedef struct {
  const uint16_t* ln1_gamma; /* [dim] (NULL = ones)  */
  const uint16_t* ln1_beta;  /* [dim] (NULL = zeros) */
  sam3_palette_linear_t qkv; /* n = 3*dim, k = dim   */
  sam3_palette_linear_t proj;/* n = dim,   k = dim   */
  const uint16_t* ln2_gamma;
  const uint16_t* ln2_beta;
  sam3_palette_linear_t fc1; /* n = hidden, k = dim  */
  sam3_palette_linear_t fc2; /* n = dim, k = hidden  */
} sam3_block_weights_t;

/* Whole-encoder weights. patch_w fp16 [dim, 3, patch, patch], patch_b [dim],
 * blocks: array of num_blocks block weights (host array of device pointers). */
typedef struct {
  const uint16_t* patch_w;
  const uint16_t* patch_b;
  const sam3_block_weights_t* blocks;
  int32_t num_blocks;
} sam3_encoder_weights_t;

/* Neck weights (fp16, device pointers): conv1 1x1 [out_dim, in_dim] (OIHW
 * with 1x1 kernels) + bias [out_dim]; conv2 3x3 [out_dim, out_dim, 3, 3] OIHW
 * + bias [out_dim]. Reference: NeckLayer.loadWeights, ViTEncoder.swift:47-52. */
typedef struct {
  const uint16_t* conv1_w;
  const uint16_t* conv1_b;
  const uint16_t* conv2_w;
  const uint16_t* conv2_b;
  int32_t in_dim;
  int32_t out_dim;
} sam3_neck_weights_t;

/* Weights of the checkpoint-faithful SAM3 encoder variant (device pointers,
 * fp16): patch_w [dim, 3, patch, patch] + patch_b [dim]; cls_token [dim] or
 * NULL (zeros, as the reference when the checkpoint has none); pos_embed
 * [1 + pos_grid^2, dim] (class position first); blocks as in
 * sam3_encoder_weights_t, any count. window: side of the attention windows in
 * tokens; the reference uses window = pos_grid (SAM3EncoderConfig.swift:45).
 * Reference: SAM3Encoder.buildGraph, SAM3Encoder.swift:280-366. */
typedef struct {
  const uint16_t* patch_w;
  const uint16_t* patch_b;
  const uint16_t* cls_token;
  const uint16_t* pos_embed;
  int32_t pos_grid;
  int32_t window;
  const sam3_block_weights_t* blocks;
  int32_t num_blocks;
} sam3_windowed_encoder_weights_t;

/* ---- context ------------------------------------------------------------ */
/* Fill *cfg with the benchmark defaults listed above. Reference: the
 * encoder topology of SAM3EncoderConfig (SAM3EncoderConfig.swift:6-12). */
sam3_status_t sam3_config_default(sam3_encoder_config_t* cfg);

/* Create a context on `device`; cfg may be NULL (defaults). Replaces the
 * per-module MTLDevice/queue set-up of ViTEncoder.init (ViTEncoder.swift:
 * 1056-1180) and the process-global CompiledGraphCache/BufferAllocator
 * (OptimizationInfrastructure.swift:20-332): the context owns one stream and a
 * workspace arena sized for cfg->max_batch, allocated up front. */
sam3_status_t sam3_ctx_create(int device, const sam3_encoder_config_t* cfg,
                              sam3_ctx_t** out);
sam3_status_t sam3_ctx_destroy(sam3_ctx_t* ctx);
/* Use a caller-provided cudaStream_t (NULL = the context's own stream), or
 * read the stream calls are queued on. Reference: the caller's
 * `commandBuffer:` every forward encodes onto (ViTEncoder.swift:374). */
sam3_status_t sam3_ctx_set_stream(sam3_ctx_t* ctx, void* cuda_stream);
void* sam3_ctx_stream(sam3_ctx_t* ctx);
/* Last error message of this context ("" when none). Never NULL.
 * Reference: the message of `SAM3Error` (SAM3MetalPipeline.swift:176). */
const char* sam3_last_error(const sam3_ctx_t* ctx);
/* Wait for the context's stream; reports device errors and kernel timeouts.
 * Reference: commandBuffer.waitUntilCompleted() (SAM3MetalPipeline.swift:79). */
sam3_status_t sam3_sync(sam3_ctx_t* ctx);
/* Count of this library's kernel launches since context creation.
 * Reference: the allocator's usage metrics (OptimizationInfrastructure.swift:
 * 230), here counting launches. */
uint64_t sam3_launch_count(const sam3_ctx_t* ctx);

/* ---- memory ---------------------------------------------------------------
 * Device buffers: BufferAllocator.privateBuffer / recycle
 * (OptimizationInfrastructure.swift:280, 307). Host-visible buffers: Apple's
 * shared-storage MTLBuffers (SAM3Predictor.swift:416) become pinned host
 * memory plus explicit copies on the context's stream that wait for
 * completion (upload / download; cf. makePrivateCopy,
 * OptimizationInfrastructure.swift:323). */
sam3_status_t sam3_alloc(sam3_ctx_t* ctx, size_t bytes, void** dptr);
sam3_status_t sam3_free(sam3_ctx_t* ctx, void* dptr);
sam3_status_t sam3_host_alloc(sam3_ctx_t* ctx, size_t bytes, void** hptr);
sam3_status_t sam3_host_free(sam3_ctx_t* ctx, void* hptr);
sam3_status_t sam3_upload(sam3_ctx_t* ctx, void* dst, const void* src, size_t bytes);
sam3_status_t sam3_download(sam3_ctx_t* ctx, void* dst, const void* src, size_t bytes);

/* ---- operators (asynchronous on the context stream) ----------------------- */

/* w_out fp16 [n, k] = palette[r, idx[r, c]] (bit-exact). Reference:
 * dequantize_int8 / dequantize_int8_optimized, Metal/Dequantize.metal:17-32,
 * 71-93 (one shared palette there; one palette per output row here). */
sam3_status_t sam3_dequant_palette(sam3_ctx_t* ctx, const sam3_palette_linear_t* w,
                                   uint16_t* w_out);

/* y fp16 [m, n] = epilogue(x [m, k] * dequant(w)^T + b), dequantization fused
 * into the tcgen05 GEMM (no dequantized weight reaches HBM). Requires
 * k % 64 == 0, n % 128 == 0, 16-byte aligned pointers.
 * residual: fp16 [m, n] for SAM3_EPI_BIAS_RESIDUAL (may equal y).
 * rope: f32 [rope_rows, 32, 2] for SAM3_EPI_BIAS_ROPE_QKV (head_dim 64,
 *   n == 3 * heads * 64); GEMM row r uses rope row (r % rope_rows).
 * Reference: the matrixMultiplication + bias calls of MPSAttentionLayer
 * (MPSAttention.swift:113-117, 179-183), MLP.forward (ViTEncoder.swift:
 * 979-997), the RoPE graph (MPSAttention.swift:137-163) and add_residual_half
 * (Metal/Common.metal:13-22, dispatched at ViTEncoder.swift:723-746). */
sam3_status_t sam3_linear_palette(sam3_ctx_t* ctx, const uint16_t* x, int32_t m,
                                  const sam3_palette_linear_t* w, int32_t epilogue,
                                  const uint16_t* residual, const float* rope,
                                  int32_t rope_rows, uint16_t* y);

/* y [m, d] = (x - mean) / sqrt(var + eps) * gamma + beta, biased variance.
 * Reference: LayerNorm.forward, ViTEncoder.swift:795-887. */
sam3_status_t sam3_layernorm(sam3_ctx_t* ctx, const uint16_t* x, int32_t m, int32_t d,
                             const uint16_t* gamma, const uint16_t* beta, float eps,
                             uint16_t* y);

/* table f32 [grid_h*grid_w, head_dim/2, 2] of (cos, sin); pairs [0, hd/4) use
 * the column index, pairs [hd/4, hd/2) the row index, freq_i = theta^(-4i/hd).
 * Reference: compute_rope_freqs_2d, Metal/RoPE.metal:22-52; RoPE.init /
 * getFrequencies, RoPE.swift:27-120. */
sam3_status_t sam3_rope_table(sam3_ctx_t* ctx, int32_t grid_h, int32_t grid_w,
                              int32_t head_dim, float theta, float* table);

/* In-place RoPE on packed qkv rows [m, 3*heads*head_dim] (q and k thirds).
 * Reference: apply_rope_2d_batch, Metal/RoPE.metal:111-153. */
sam3_status_t sam3_rope_apply(sam3_ctx_t* ctx, uint16_t* qkv, int32_t m, int32_t heads,
                              int32_t head_dim, const float* table, int32_t rope_rows);

/* o [batch*seq, heads*64] = softmax(q k^T * scale) v per image and head, from
 * packed rows qkv [batch*seq, 3*heads*64]. Global (unmasked) attention.
 * Reference: scaledDotProductAttention, MPSAttention.swift:165-176;
 * AttentionKernels.referenceSoftmax, AttentionKernels.swift:48-68. */
sam3_status_t sam3_attention(sam3_ctx_t* ctx, const uint16_t* qkv, int32_t batch,
                             int32_t seq, int32_t heads, int32_t head_dim, float scale,
                             uint16_t* o);

/* Capacity of sam3_prune_noalloc's fixed score scratch (batch * seq rows). */
#define SAM3_PRUNE_NOALLOC_MAX_ROWS 65536

/* sam3_prune without a context and without allocating anything: the same
 * scoring, selection (ties to the lower index) and gather, enqueued on
 * `cuda_stream` (a cudaStream_t; NULL = the legacy default stream).
 * No counterpart in the reference; it exists for callers that cannot
 * allocate device memory: code that runs inside a host application owning
 * every device allocation under a fixed budget, threads that must not call
 * cudaMalloc / cudaFree because those calls can block or synchronise the
 * device, and callers with no sam3 context (creating one allocates its
 * workspace). Such a caller passes its own input and output buffers; the
 * per-token score scratch is a fixed 256 KB device array inside the library
 * (SAM3_PRUNE_NOALLOC_MAX_ROWS floats, held on every GPU that loads the
 * library until the process exits). batch * seq beyond that limit returns
 * SAM3_ERR_SHAPE; other argument errors return SAM3_ERR_INVALID_ARG /
 * SAM3_ERR_SHAPE as sam3_prune does, and a failed launch SAM3_ERR_CUDA.
 * The work runs on the stream's device, which is made current for the call
 * (the calling thread's current device is restored before returning). An
 * error already pending on the calling thread is left in place, not cleared.
 * The first call on each device looks up the array's device address (and
 * raises the selection kernel's shared-memory limit there), so make it
 * before any stream capture. That address is kept for the life of the
 * process: after cudaDeviceReset of a device, do not call this entry point
 * on that device again. All calls share the one array: calls that overlap on
 * the GPU (different streams, or graph replays running at the same time)
 * race on it and must be serialised by the caller. */
sam3_status_t sam3_prune_noalloc(void* cuda_stream, const uint16_t* x, int32_t batch,
                                 int32_t seq, int32_t d, int32_t keep, int32_t norm,
                                 int32_t order, const float* rope_in, int32_t rope_rows,
                                 int32_t rope_cols, uint16_t* feats, float* rope_out,
                                 int32_t* idx);

/* Token scores f32 [rows] = L2 norm or L1 (sum |x|) of each row.
 * Reference: TokenPruner.swift:54-56. */
sam3_status_t sam3_token_scores(sam3_ctx_t* ctx, const uint16_t* x, int32_t rows,
                                int32_t d, int32_t norm, float* scores);

/* Prune each image of x [batch*seq, d] to its `keep` highest-scoring tokens
 * (ties to the lower index), in ascending index order (SAM3_ORDER_INDEX) or by
 * descending score (SAM3_ORDER_SCORE). Outputs: feats fp16 [batch*keep, d],
 * rope_out f32 [batch*keep, rope_cols] gathered from rope_in row
 * ((b*seq + token) % rope_rows) (rope_in/rope_out may be NULL), idx int32
 * [batch, keep] (token index within its image). seq <= 16384.
 * Reference: TokenPruner.prune, TokenPruner.swift:32-126. */
sam3_status_t sam3_prune(sam3_ctx_t* ctx, const uint16_t* x, int32_t batch, int32_t seq,
                         int32_t d, int32_t keep, int32_t norm, int32_t order,
                         const float* rope_in, int32_t rope_rows, int32_t rope_cols,
                         uint16_t* feats, float* rope_out, int32_t* idx);

/* Patch embedding: NHWC fp16 image [batch, h, w, 3] -> tokens [batch*gh*gw, dim]
 * (row-major h*gw + w), conv weights fp16 [dim, 3, patch, patch], bias [dim].
 * Reference: PatchEmbedding.forward, ViTEncoder.swift:218-263, and the flatten
 * kernel texture_to_buffer_flat_half, Metal/ViTUtils.metal:53-76. */
sam3_status_t sam3_patch_embed(sam3_ctx_t* ctx, const uint16_t* image, int32_t batch,
                               int32_t height, int32_t width, const uint16_t* patch_w,
                               const uint16_t* patch_b, int32_t patch, int32_t dim,
                               uint16_t* out);

/* Camera-frame preprocessing: f32 RGBA [batch, height, width, 4] with values
 * in [0, 1] -> fp16 RGB [batch, height, width, 3] = (rgb - mean) / std with
 * the ImageNet mean (0.485, 0.456, 0.406) and std (0.229, 0.224, 0.225), in
 * fp32 with IEEE division, rounded to fp16; alpha is dropped. rgba 16-byte
 * aligned. Reference: SAM3Predictor.setImage, the slice_rgb / sub_mean /
 * div_std nodes, SAM3Predictor.swift:332-341. */
sam3_status_t sam3_preprocess_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch,
                                   int32_t height, int32_t width, uint16_t* rgb);

/* Patch embedding straight from f32 RGBA frames: the preprocessing above is
 * applied while the patches are gathered, so the normalised image never
 * exists in memory. Output equals sam3_patch_embed on sam3_preprocess_rgba's
 * output, bit for bit. Reference: SAM3Predictor.swift:332-341 followed by
 * PatchEmbedding.forward, ViTEncoder.swift:218-263. */
sam3_status_t sam3_patch_embed_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch,
                                    int32_t height, int32_t width, const uint16_t* patch_w,
                                    const uint16_t* patch_b, int32_t patch, int32_t dim,
                                    uint16_t* out);

/* x [batch*seq, dim] -> x + attn(LN1(x)) (in place). Reference: LN1 +
 * MPSAttentionLayer.forward + residual of TransformerBlock.forward,
 * ViTEncoder.swift:388-411; MPSAttention.swift:85-244. */
sam3_status_t sam3_attention_block(sam3_ctx_t* ctx, uint16_t* x, int32_t batch,
                                   int32_t seq, const sam3_block_weights_t* w,
                                   const float* rope, int32_t rope_rows);

/* x [m, dim] -> x + MLP(LN2(x)) (in place). Reference: LN2 + MLP.forward +
 * residual, ViTEncoder.swift:412-430, 953-1050. */
sam3_status_t sam3_mlp_block(sam3_ctx_t* ctx, uint16_t* x, int32_t m,
                             const sam3_block_weights_t* w);

/* One pre-LN ViT block in place on x [batch*seq, dim]; rope f32
 * [rope_rows, 32, 2], GEMM row r uses rope row r % rope_rows. Reference:
 * TransformerBlock.forward, ViTEncoder.swift:368-431 (fused form :433-691). */
sam3_status_t sam3_vit_block(sam3_ctx_t* ctx, uint16_t* x, int32_t batch, int32_t seq,
                             const sam3_block_weights_t* w, const float* rope,
                             int32_t rope_rows);

/* Full encoder on device buffers: image fp16 NHWC [batch, S, S, 3] ->
 * feats fp16 [batch, keep, dim] (or [batch, seq, dim] without pruning) and
 * idx int32 [batch, keep] (token index of each kept row). batch <= max_batch.
 * Reference: ViTEncoder.forward(image:commandBuffer:), ViTEncoder.swift:
 * 1235-1481. */
sam3_status_t sam3_encoder_forward(sam3_ctx_t* ctx, const uint16_t* image, int32_t batch,
                                   const sam3_encoder_weights_t* w, uint16_t* feats,
                                   int32_t* idx);

/* Full encoder from f32 RGBA camera frames [batch, S, S, 4] in [0, 1] on the
 * device: the ImageNet normalisation is fused into the patch embedding (see
 * sam3_patch_embed_rgba); otherwise as sam3_encoder_forward. Reference:
 * SAM3Predictor.setImage's preprocessing (SAM3Predictor.swift:332-341) feeding
 * ViTEncoder.forward (ViTEncoder.swift:1235-1481). */
sam3_status_t sam3_encoder_forward_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch,
                                        const sam3_encoder_weights_t* w, uint16_t* feats,
                                        int32_t* idx);

/* Same, from and to HOST buffers (pinned or pageable): copies the images in,
 * runs the encoder and copies feats/idx out, then waits. Reference:
 * SAM3MetalPipeline.encode(image:), SAM3MetalPipeline.swift:67-82. */
sam3_status_t sam3_encoder_forward_host(sam3_ctx_t* ctx, const uint16_t* host_image,
                                        int32_t batch, const sam3_encoder_weights_t* w,
                                        uint16_t* host_feats, int32_t* host_idx);

/* Any number of images from and to HOST buffers, in chunks of max_batch,
 * with the copies overlapped: while the encoder runs on chunk c, a copy
 * stream uploads chunk c+1's images and downloads chunk c-1's features and
 * indices (double-buffered device staging, allocated on first use: about
 * 2 x max_batch x (image + features) bytes). host_image [n_images, S, S, 3]
 * fp16, host_feats [n_images, out_tokens, dim] fp16, host_idx
 * [n_images, out_tokens] int32; the results equal sam3_encoder_forward_host's
 * bit for bit. Returns when everything is on the host. Pinned host memory is
 * needed for the copies to overlap (pageable memory works, serialised).
 * Reference: the per-batch encode + host gather of SAM3MetalPipeline
 * (SAM3MetalPipeline.swift:67-82), here overlapped with the next batch. */
sam3_status_t sam3_encoder_forward_host_pipelined(sam3_ctx_t* ctx, const uint16_t* host_image,
                                                  int32_t n_images,
                                                  const sam3_encoder_weights_t* w,
                                                  uint16_t* host_feats, int32_t* host_idx);

/* The same work without the wait: enqueues the uploads, the encoder and the
 * downloads of n_images and returns at once with a ticket (1, 2, ... per
 * context). Uploads and downloads run on their own streams, so a later
 * submission's uploads overlap this one's encoder and this one's downloads
 * overlap the next encoder: a stream of frames keeps the GPU busy across
 * calls. The host buffers must stay valid, and host_feats/host_idx unread,
 * until sam3_encoder_wait_host(ticket) returns SAM3_OK. Keep the context's
 * stream unchanged while submissions are in flight. Reference: the encoder
 * recorded into a command buffer and committed, SAM3MetalPipeline.swift:72-77
 * (ViTEncoder.forward(image:commandBuffer:) + commandBuffer.commit()). */
sam3_status_t sam3_encoder_submit_host(sam3_ctx_t* ctx, const uint16_t* host_image,
                                       int32_t n_images, const sam3_encoder_weights_t* w,
                                       uint16_t* host_feats, int32_t* host_idx,
                                       uint64_t* ticket);

/* Blocks until the downloads of submission `ticket` (and of every earlier
 * one) are on the host. SAM3_ERR_INVALID_ARG for a ticket not issued;
 * SAM3_ERR_TIMEOUT / SAM3_ERR_INVALID_ARG when the device error word was set
 * by the time that submission's encoder ended (the word stays set until
 * sam3_sync reads and clears it). Reference: commandBuffer.waitUntilCompleted(),
 * SAM3MetalPipeline.swift:79. */
sam3_status_t sam3_encoder_wait_host(sam3_ctx_t* ctx, uint64_t ticket);

/* Pruned rows back to their grid positions: out [batch, seq, dim] fp16 is
 * zero except out[b, idx[b, k], :] = pruned[b, k, :] (idx int32 [batch, keep],
 * unique per image, as sam3_prune writes them). An index outside [0, seq) is
 * skipped and reported by the next sam3_sync as SAM3_ERR_INVALID_ARG. dim % 8
 * == 0. Reference: TokenPruner.restoreSpatial, TokenPruner.swift:130-196. */
sam3_status_t sam3_restore_spatial(sam3_ctx_t* ctx, const uint16_t* pruned, const int32_t* idx,
                                   int32_t batch, int32_t keep, int32_t seq, int32_t dim,
                                   uint16_t* out);

/* FPN-style neck on x fp16 [batch, height*width, in_dim] (row-major grid):
 * conv 1x1 in_dim -> out_dim + bias, then conv 3x3 (padding 1) out_dim ->
 * out_dim + bias, NHWC fp16 out [batch, height, width, out_dim]; fp16 between
 * the convs, fp32 accumulation. in_dim % 64 == 0, out_dim % 128 == 0, and the
 * grid must fit the context workspace (batch*height*width <= max_batch *
 * tokens per image). Reference: NeckLayer.forward, ViTEncoder.swift:54-140. */
sam3_status_t sam3_neck(sam3_ctx_t* ctx, const uint16_t* x, int32_t batch, int32_t height,
                        int32_t width, const sam3_neck_weights_t* w, uint16_t* out);

/* Checkpoint-faithful SAM3 encoder on fp16 RGB images [batch, S, S, 3] (S =
 * image_size of the config; embed_dim, num_heads, mlp_hidden, ln_eps and
 * rope_theta from the config too): patch embedding, class token prepended,
 * pos_embed added (class position, then the pos_grid^2 table resized to the
 * token grid by bilinear interpolation with half-pixel centres), then the
 * blocks: block i attends globally when i % stride == stride - 1 (stride =
 * max(1, num_blocks / 4)), else inside window x window token windows without
 * the class token (whose attention output is zero); RoPE (the grid table)
 * rotates the patch tokens only. out fp16 [batch, grid*grid, dim], grid
 * order, class token dropped, no pruning. window must divide the grid.
 * Reference: SAM3Encoder.buildGraph / buildTransformerBlock /
 * buildFusedQKVAttention, SAM3Encoder.swift:280-366, 368-460, 545-720. */
sam3_status_t sam3_windowed_encoder_forward(sam3_ctx_t* ctx, const uint16_t* image,
                                            int32_t batch,
                                            const sam3_windowed_encoder_weights_t* w,
                                            uint16_t* out);

/* Same from f32 RGBA camera frames [batch, S, S, 4] in [0, 1] on the device,
 * the ImageNet normalisation fused into the patch embedding (as
 * sam3_encoder_forward_rgba). Reference: SAM3Predictor.setImage's
 * preprocessing (SAM3Predictor.swift:332-341) feeding SAM3Encoder's graph
 * (SAM3Encoder.swift:259-366). */
sam3_status_t sam3_windowed_encoder_forward_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch,
                                                 const sam3_windowed_encoder_weights_t* w,
                                                 uint16_t* out);

/* ---- failure detection and fault injection ------------------------------
 * Every wait inside a kernel (mbarriers of the TMA / MMA pipelines) is bounded
 * (2 s); on expiry the kernel records a code in the context's device error
 * word, drains its copies in flight and returns, and the next sam3_sync
 * returns SAM3_ERR_TIMEOUT and clears the word: the context stays usable.
 * Reference: errors surface as `throws SAM3Error`
 * (SAM3MetalPipeline.swift:176-208); it has no device-side watchdog. */

/* Launches a one-thread kernel whose bounded wait, on an mbarrier nothing
 * arrives on, runs out: the following sam3_sync returns SAM3_ERR_TIMEOUT
 * (after about 2 s) without any GPU fault. */
sam3_status_t sam3_selftest_wait_timeout(sam3_ctx_t* ctx);

/* Host-side fault injection for the error paths (no GPU fault is made):
 * SAM3_FAULT_ALLOC makes sam3_alloc, sam3_host_alloc and the staging
 * allocation of sam3_encoder_forward_host_pipelined fail with SAM3_ERR_OOM;
 * SAM3_FAULT_LAUNCH makes every kernel-launch check report SAM3_ERR_CUDA
 * (the kernel itself may have run). The environment variable SAM3_FAULT
 * ("alloc", "launch", "alloc,launch") sets the flags of every new context. */
typedef enum { SAM3_FAULT_NONE = 0, SAM3_FAULT_ALLOC = 1, SAM3_FAULT_LAUNCH = 2 } sam3_fault_t;
sam3_status_t sam3_set_fault(sam3_ctx_t* ctx, int32_t flags);
int32_t sam3_get_fault(const sam3_ctx_t* ctx);

/* ---- device-side stage timing ---------------------------------------------
 * When enabled, the context brackets each of its kernel launches with CUDA
 * events on its stream and accumulates, per kernel class, the launch count,
 * the device time and the algorithmic work (GEMM and attention FLOPs, bytes of
 * the memory-bound kernels). Reference: the SAM3_STAGE_TIMING stage timer of
 * ViTEncoder.forward (ViTEncoder.swift:1236-1237,1438-1450; Sam3Log.swift:
 * 9-25), which timed CPU encode time; this one times the device. */
typedef enum {
  SAM3_PROF_GEMM = 0,      /* palette-dequant GEMMs (QKV, proj, fc1, fc2)   */
  SAM3_PROF_ATTENTION = 1, /* softmax attention                             */
  SAM3_PROF_LAYERNORM = 2,
  SAM3_PROF_PRUNE = 3,     /* scores + select + gather                      */
  SAM3_PROF_PATCH = 4,     /* im2col + weight pad + dense patch GEMM        */
  SAM3_PROF_OTHER = 5,     /* RoPE table/apply, dequant, iota               */
  SAM3_PROF_CLASSES = 6
} sam3_prof_class_t;

typedef struct {
  uint64_t launches[SAM3_PROF_CLASSES];
  double milliseconds[SAM3_PROF_CLASSES]; /* summed device time of launches */
  double flops[SAM3_PROF_CLASSES];        /* 2*m*n*k (GEMM), 4*B*H*S^2*d    */
  double bytes[SAM3_PROF_CLASSES];        /* algorithmic HBM bytes          */
} sam3_profile_t;

/* Turn timing on (resets the counters) or off. */
sam3_status_t sam3_profile_enable(sam3_ctx_t* ctx, int32_t enable);
/* Wait for the stream and return the counters accumulated since enabling. */
sam3_status_t sam3_profile_read(sam3_ctx_t* ctx, sam3_profile_t* out);

/* Rows kept per image by the encoder under the context's config: keep_tokens
 * when the config prunes, else the full grid. Reference: the kept count of
 * TokenPruner.prune (TokenPruner.swift:32-126). */
int32_t sam3_encoder_out_tokens(const sam3_ctx_t* ctx);

#ifdef __cplusplus
}
#endif
#endif /* SAM3CUDA_H */
