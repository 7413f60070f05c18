// sam3_modules.hpp - C++ host-side mirror of the reference's operator classes
// for the encoder hot path, over the C ABI of libsam3cuda (header-only).
//
// The reference exposes these as Swift classes (OrdoSAM3Sensor/Sources/
// Sam3Sensor): RoPE (RoPE.swift:9-121), LayerNorm (ViTEncoder.swift:751-888),
// MLP (ViTEncoder.swift:892-1051), MPSAttentionLayer (MPSAttention.swift:
// 13-244), TransformerBlock (ViTEncoder.swift:299-747), TokenPruner
// (TokenPruner.swift:11-197), ViTEncoder (ViTEncoder.swift:1056-1481) and
// the checkpoint-faithful SAM3Encoder (SAM3Encoder.swift:10-760).
// The classes below keep their names, method names and argument meaning:
//  - `forward(...)` returns a freshly allocated device buffer and appends it
//    to `recycledBuffers`, as the reference does with BufferAllocator
//    (the caller frees them once the stream has finished: recycle());
//  - errors throw sam3::SAM3Error (the reference's `throws SAM3Error`);
//  - `commandBuffer` becomes the context's CUDA stream;
//  - `windowed` is accepted and ignored: every block attends globally, as
//    MPSAttentionLayer does (it forces sEff = seqLen, MPSAttention.swift:97-104).
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/sam3cuda.h"

namespace sam3 {

struct SAM3Error : std::runtime_error {
  sam3_status_t status;
  SAM3Error(sam3_status_t s, const std::string& what) : std::runtime_error(what), status(s) {}
};

inline void check(sam3_ctx_t* ctx, sam3_status_t st, const char* where) {
  if (st != SAM3_OK)
    throw SAM3Error(st, std::string(where) + ": " + (ctx ? sam3_last_error(ctx) : "no context"));
}

using BufferList = std::vector<void*>;

inline void* allocate(sam3_ctx_t* ctx, size_t bytes, BufferList& recycled, const char* what) {
  void* p = nullptr;
  check(ctx, sam3_alloc(ctx, bytes, &p), what);
  recycled.push_back(p);
  return p;
}

// Frees every buffer a forward() handed out, after the stream has drained
// (the reference recycles in the command buffer's completion handler,
// ViTEncoder.swift:1459-1464). The buffers are freed even when the sync
// reports an error (a kernel timeout leaves the context usable); the error
// is thrown afterwards.
inline void recycle(sam3_ctx_t* ctx, BufferList& recycled) {
  const sam3_status_t st = sam3_sync(ctx);
  for (void* p : recycled) sam3_free(ctx, p);
  recycled.clear();
  check(ctx, st, "recycle sync");
}

// RoPE.swift:9-121: the 2D axial table for a square grid, built once.
class RoPE {
 public:
  RoPE(sam3_ctx_t* ctx, int maxSeqLen, int headDim = 64, float theta = 10000.0f) : ctx_(ctx) {
    int side = 0;
    while ((side + 1) * (side + 1) <= maxSeqLen) ++side;
    if (side * side != maxSeqLen)  // RoPE.swift:86-90 precondition
      throw SAM3Error(SAM3_ERR_SHAPE, "RoPE: maxSeqLen is not a perfect square");
    check(ctx, sam3_alloc(ctx, (size_t)maxSeqLen * headDim * sizeof(float), &table_), "RoPE alloc");
    check(ctx, sam3_rope_table(ctx, side, side, headDim, theta, static_cast<float*>(table_)),
          "RoPE table");
    seq_ = maxSeqLen;
  }
  ~RoPE() {
    if (table_) sam3_free(ctx_, table_);
  }
  RoPE(const RoPE&) = delete;
  RoPE& operator=(const RoPE&) = delete;
  const float* getFrequencies() const { return static_cast<const float*>(table_); }
  int rows() const { return seq_; }

 private:
  sam3_ctx_t* ctx_;
  void* table_ = nullptr;
  int seq_ = 0;
};

// ViTEncoder.swift:751-888.
class LayerNorm {
 public:
  LayerNorm(sam3_ctx_t* ctx, int dim, const uint16_t* gamma = nullptr,
            const uint16_t* beta = nullptr, float eps = 1e-6f)
      : ctx_(ctx), dim_(dim), gamma_(gamma), beta_(beta), eps_(eps) {}
  uint16_t* forward(const uint16_t* input, int seqLen, int batch, BufferList& recycledBuffers) {
    const int m = seqLen * batch;
    auto* out = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)m * dim_ * 2, recycledBuffers, "LayerNorm output"));
    check(ctx_, sam3_layernorm(ctx_, input, m, dim_, gamma_, beta_, eps_, out), "LayerNorm");
    return out;
  }

 private:
  sam3_ctx_t* ctx_;
  int dim_;
  const uint16_t *gamma_, *beta_;
  float eps_;
};

// ViTEncoder.swift:892-1051 (fc1 + bias + erf GELU + fc2 + bias); the
// residual add of the block (ViTEncoder.swift:412-430) is TransformerBlock's.
class MLP {
 public:
  MLP(sam3_ctx_t* ctx, int inputDim, int hiddenDim)
      : ctx_(ctx), in_(inputDim), hidden_(hiddenDim) {}
  void loadWeights(const sam3_palette_linear_t& fc1, const sam3_palette_linear_t& fc2) {
    fc1_ = fc1;
    fc2_ = fc2;
  }
  uint16_t* forward(const uint16_t* input, int seqLen, int batch, BufferList& recycledBuffers) {
    const int m = seqLen * batch;
    auto* h = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)m * hidden_ * 2, recycledBuffers, "MLP hidden"));
    auto* out = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)m * in_ * 2, recycledBuffers, "MLP output"));
    check(ctx_, sam3_linear_palette(ctx_, input, m, &fc1_, SAM3_EPI_BIAS_GELU, nullptr, nullptr,
                                    0, h),
          "MLP fc1");
    check(ctx_, sam3_linear_palette(ctx_, h, m, &fc2_, SAM3_EPI_BIAS, nullptr, nullptr, 0, out),
          "MLP fc2");
    return out;
  }

 private:
  sam3_ctx_t* ctx_;
  int in_, hidden_;
  sam3_palette_linear_t fc1_{}, fc2_{};
};

// MPSAttention.swift:13-244: QKV (+bias) -> RoPE(q, k) -> SDPA -> proj (+bias).
class MPSAttentionLayer {
 public:
  MPSAttentionLayer(sam3_ctx_t* ctx, int dim, int numHeads)
      : ctx_(ctx), dim_(dim), heads_(numHeads) {}
  void loadWeights(const sam3_palette_linear_t& qkv, const sam3_palette_linear_t& proj) {
    qkv_ = qkv;
    proj_ = proj;
  }
  uint16_t* forward(const uint16_t* input, const float* ropeFreqs, int batch, int seqLen,
                    bool windowed, BufferList& recycledBuffers, int ropeRows = 0) {
    (void)windowed;
    const int m = seqLen * batch;
    auto* qkv = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)m * 3 * dim_ * 2, recycledBuffers, "attention qkv"));
    auto* att = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)m * dim_ * 2, recycledBuffers, "attention out"));
    auto* out = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)m * dim_ * 2, recycledBuffers, "attention proj"));
    check(ctx_, sam3_linear_palette(ctx_, input, m, &qkv_, SAM3_EPI_BIAS_ROPE_QKV, nullptr,
                                    ropeFreqs, ropeRows > 0 ? ropeRows : seqLen, qkv),
          "attention qkv");
    check(ctx_, sam3_attention(ctx_, qkv, batch, seqLen, heads_, dim_ / heads_, 0.125f, att),
          "attention sdpa");
    check(ctx_, sam3_linear_palette(ctx_, att, m, &proj_, SAM3_EPI_BIAS, nullptr, nullptr, 0, out),
          "attention proj");
    return out;
  }

 private:
  sam3_ctx_t* ctx_;
  int dim_, heads_;
  sam3_palette_linear_t qkv_{}, proj_{};
};

// ViTEncoder.swift:299-747: x + attn(LN1(x)), then + MLP(LN2(.)); fused on
// the device (residuals in the GEMM epilogues), one output buffer per call.
class TransformerBlock {
 public:
  TransformerBlock(sam3_ctx_t* ctx, int dim, int numHeads, int mlpHiddenDim)
      : ctx_(ctx), dim_(dim), heads_(numHeads), hidden_(mlpHiddenDim) {}
  void loadWeights(const sam3_block_weights_t& w) { w_ = w; }
  uint16_t* forward(const uint16_t* input, const float* ropeFreqs, int seqLen, int batch,
                    bool windowed, BufferList& recycledBuffers, int ropeRows = 0) {
    (void)windowed;
    const size_t bytes = (size_t)seqLen * batch * dim_ * 2;
    auto* out = static_cast<uint16_t*>(allocate(ctx_, bytes, recycledBuffers, "block output"));
    cudaStream_t s = static_cast<cudaStream_t>(sam3_ctx_stream(ctx_));
    if (cudaMemcpyAsync(out, input, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      throw SAM3Error(SAM3_ERR_CUDA, "TransformerBlock: input copy failed");
    check(ctx_, sam3_vit_block(ctx_, out, batch, seqLen, &w_, ropeFreqs,
                               ropeRows > 0 ? ropeRows : seqLen),
          "TransformerBlock");
    return out;
  }

 private:
  sam3_ctx_t* ctx_;
  int dim_, heads_, hidden_;
  sam3_block_weights_t w_{};
};

// TokenPruner.swift:11-197. prune() returns (features, RoPE rows, indices).
// The reference scores with L1 and orders by score (MPSGraph topK); the
// defaults here follow the benchmark spec (L2, ascending token index).
class TokenPruner {
 public:
  TokenPruner(sam3_ctx_t* ctx, int keepK, int dim, int ropeDim = 64,
              int norm = SAM3_SCORE_L2, int order = SAM3_ORDER_INDEX)
      : ctx_(ctx), keep_(keepK), dim_(dim), rope_dim_(ropeDim), norm_(norm), order_(order) {}
  std::tuple<uint16_t*, float*, int32_t*> prune(const uint16_t* input, const float* ropeFreqs,
                                                int seqLen, int batch,
                                                BufferList& recycledBuffers) {
    auto* feats = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)batch * keep_ * dim_ * 2, recycledBuffers, "PrunedFeats"));
    auto* rope = static_cast<float*>(
        allocate(ctx_, (size_t)batch * keep_ * rope_dim_ * 4, recycledBuffers, "PrunedRoPE"));
    auto* idx = static_cast<int32_t*>(
        allocate(ctx_, (size_t)batch * keep_ * 4, recycledBuffers, "PruneIndices"));
    check(ctx_, sam3_prune(ctx_, input, batch, seqLen, dim_, keep_, norm_, order_, ropeFreqs,
                           seqLen, rope_dim_, feats, rope, idx),
          "TokenPruner.prune");
    return {feats, rope, idx};
  }

 private:
  sam3_ctx_t* ctx_;
  int keep_, dim_, rope_dim_, norm_, order_;
};

// ViTEncoder.swift:1056-1481: image -> pruned token features (+ indices).
class ViTEncoder {
 public:
  ViTEncoder(sam3_ctx_t* ctx, const sam3_encoder_weights_t& w, int embedDim = 1024)
      : ctx_(ctx), w_(w), dim_(embedDim) {}
  // image: device fp16 NHWC [batch, S, S, 3]. Returns feats [batch, keep, dim];
  // the kept token indices [batch, keep] go to *indices. Both buffers are
  // appended to recycledBuffers.
  uint16_t* forward(const uint16_t* image, int batch, BufferList& recycledBuffers,
                    int32_t** indices = nullptr) {
    const int keep = sam3_encoder_out_tokens(ctx_);
    auto* idx = static_cast<int32_t*>(
        allocate(ctx_, (size_t)batch * keep * 4, recycledBuffers, "encoder indices"));
    auto* feats = static_cast<uint16_t*>(
        allocate(ctx_, (size_t)batch * keep * dim_ * 2, recycledBuffers, "encoder features"));
    check(ctx_, sam3_encoder_forward(ctx_, image, batch, &w_, feats, idx), "ViTEncoder.forward");
    if (indices) *indices = idx;
    return feats;
  }

  // Many images from and to host memory (SAM3MetalPipeline.encode,
  // SAM3MetalPipeline.swift:67-82, over a whole set of frames): chunks of
  // max_batch with the copies overlapped; returns when all are on the host.
  void encodeHost(const uint16_t* hostImages, int nImages, uint16_t* hostFeats,
                  int32_t* hostIndices) {
    check(ctx_, sam3_encoder_forward_host_pipelined(ctx_, hostImages, nImages, &w_, hostFeats,
                                                    hostIndices),
          "ViTEncoder.encodeHost");
  }

  // The same, committed without waiting (SAM3MetalPipeline.swift:72-77, the
  // encoder recorded into a command buffer and committed): returns a ticket;
  // waitHost(ticket) is waitUntilCompleted (:79). Buffers stay owned by the
  // caller and untouched until then.
  uint64_t submitHost(const uint16_t* hostImages, int nImages, uint16_t* hostFeats,
                      int32_t* hostIndices) {
    uint64_t ticket = 0;
    check(ctx_, sam3_encoder_submit_host(ctx_, hostImages, nImages, &w_, hostFeats, hostIndices,
                                         &ticket),
          "ViTEncoder.submitHost");
    return ticket;
  }
  void waitHost(uint64_t ticket) {
    check(ctx_, sam3_encoder_wait_host(ctx_, ticket), "ViTEncoder.waitHost");
  }

 private:
  sam3_ctx_t* ctx_;
  sam3_encoder_weights_t w_;
  int dim_;
};

// SAM3Encoder.swift:10-760: class token, resized positional embedding,
// windowed blocks with global ones every num_blocks / 4; returns the patch
// tokens [batch, grid*grid, dim] in grid order.
class SAM3Encoder {
 public:
  SAM3Encoder(sam3_ctx_t* ctx, const sam3_windowed_encoder_weights_t& w, int embedDim = 1024,
              int gridSize = 72)
      : ctx_(ctx), w_(w), dim_(embedDim), grid_(gridSize) {}
  uint16_t* forward(const uint16_t* image, int batch, BufferList& recycledBuffers) {
    auto* out = static_cast<uint16_t*>(allocate(ctx_, (size_t)batch * grid_ * grid_ * dim_ * 2,
                                                recycledBuffers, "SAM3Encoder output"));
    check(ctx_, sam3_windowed_encoder_forward(ctx_, image, batch, &w_, out),
          "SAM3Encoder.forward");
    return out;
  }

 private:
  sam3_ctx_t* ctx_;
  sam3_windowed_encoder_weights_t w_;
  int dim_, grid_;
};

}  // namespace sam3
