// internal.h - context object and internal launchers shared by the .cu files
// of libsam3cuda. Not part of the public ABI (include/sam3cuda.h is).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/sam3cuda.h"

struct sam3_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;  // the stream operators run on
  sam3_encoder_config_t cfg{};
  std::string last_error;
  int* dev_err = nullptr;  // device error word written by bounded waits
  uint64_t launches = 0;
  int fault = 0;  // SAM3_FAULT_* flags: host-side fault injection for tests

  // Workspace arena (allocated at create, sized for cfg.max_batch images).
  char* ws = nullptr;
  size_t ws_bytes = 0;
  size_t ws_used = 0;
  // Encoder scratch carved from the arena.
  uint16_t* x = nullptr;        // [B*S, D] residual stream
  uint16_t* xp = nullptr;       // [B*keep, D] residual stream after pruning
  uint16_t* ln = nullptr;       // [B*S, D]
  uint16_t* qkv = nullptr;      // [B*S, 3D]
  uint16_t* attn = nullptr;     // [B*S, D]
  uint16_t* hidden = nullptr;   // [B*S, F]
  uint16_t* cols = nullptr;     // [B*S, Kp] im2col of the patch embedding
  uint16_t* patch_wp = nullptr; // [D, Kp] padded patch weights
  float* scores = nullptr;      // [B*S]
  float* rope = nullptr;        // [S, 32, 2]
  float* rope_pruned = nullptr; // [B*keep, 32, 2]
  // Axial form of the grid table for the QKV GEMM epilogue, pair-major:
  // float4 [q][c] = pairs 2q, 2q+1 at coordinate c (q < 8, c < grid); per row
  // the coordinates x | y << 16.
  float* rope_axial = nullptr;        // [8, grid, 4]
  int32_t* rope_pos_grid = nullptr;   // [B*S] grid order
  int32_t* rope_pos_win = nullptr;    // [B*(S+1)] window-major, -1 for the class token
  int32_t* rope_pos_pruned = nullptr; // [B*keep] the kept tokens
  int rope_win_key = 0;               // window size rope_pos_win was built for (0: none)
  int32_t* idx = nullptr;       // [B*keep]
  uint16_t* image = nullptr;    // [B, H, W, 3] staging for the host API
  uint16_t* feats = nullptr;    // [B*keep, D] staging for the host API
  int rope_ready = 0;
  // Block-level scratch used by sam3_vit_block & co. outside the encoder.
  size_t block_rows = 0;        // rows the block scratch can hold (plain encoder)
  size_t token_rows = 0;        // rows with a class token per image (windowed encoder)

  // Double-buffered staging of the host-buffer encoder submissions
  // (sam3_encoder_submit_host and the calls built on it), made on first use:
  // two sets of (images, features, indices), an upload and a download stream.
  cudaStream_t copy_stream = nullptr;  // uploads
  cudaStream_t down_stream = nullptr;  // downloads
  char* pipe_mem = nullptr;
  size_t pipe_bytes = 0;
  cudaEvent_t pipe_ev[8] = {};  // in_done[2], img_free[2], out_ready[2], out_done[2]
  uint64_t pipe_chunks = 0;     // chunks issued so far; chunk g uses staging set g & 1
  // Submission tickets (1, 2, ...): the last kPipeTickets keep an event on
  // the download stream and a pinned copy of the device error word, both
  // taken after the submission's last download.
  static constexpr int kPipeTickets = 8;
  uint64_t pipe_tickets = 0;
  cudaEvent_t pipe_done[kPipeTickets] = {};
  int* pipe_err = nullptr;      // pinned host [kPipeTickets]

  // Device-side stage timing (sam3_profile_enable / sam3_profile_read).
  struct ProfRecord {
    int cls;
    double flops, bytes;
    cudaEvent_t start, stop;
  };
  bool profiling = false;
  std::vector<ProfRecord> prof_pending;
  std::vector<cudaEvent_t> event_pool;
  sam3_profile_t prof{};

  // Kernels whose dynamic shared-memory limit has been raised on this
  // context's device (sam3::kSmem* bits; the attribute is per device).
  uint32_t smem_attr_done = 0;
};

namespace sam3 {

sam3_status_t set_error(sam3_ctx_t* ctx, sam3_status_t code, const char* fmt, ...);
sam3_status_t check_launch(sam3_ctx_t* ctx, const char* what);
// For launches that return their error (cudaLaunchKernelEx).
sam3_status_t check_launch_ret(sam3_ctx_t* ctx, cudaError_t e, const char* what);
sam3_status_t check_cuda(sam3_ctx_t* ctx, cudaError_t e, const char* what);
// Status for a value of the device error word (0: SAM3_OK), with the message.
sam3_status_t device_error_status(sam3_ctx_t* ctx, int err);

// Raise `kernel`'s dynamic shared-memory limit to `bytes` once per context:
// the attribute belongs to the device, and each context is bound to one.
enum : uint32_t {
  kSmemAttn = 1u, kSmemWs = 2u, kSmemWsc = 4u, kSmemGemm = 8u /* << MODE */, kSmemPrune = 64u,
  kSmemAttnPP = 128u
};
template <typename Kernel>
sam3_status_t ensure_smem_attr(sam3_ctx_t* ctx, uint32_t bit, Kernel kernel, int bytes,
                               const char* what) {
  if (ctx->smem_attr_done & bit) return SAM3_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return check_cuda(ctx, e, what);
  ctx->smem_attr_done |= bit;
  return SAM3_OK;
}
sam3_status_t ensure_workspace(sam3_ctx_t* ctx);
bool aligned16(const void* p);

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();

// Launchers (validate, then enqueue on ctx->stream).
sam3_status_t gemm_palette(sam3_ctx_t* ctx, const uint16_t* x, int m, int k,
                           const uint8_t* idx, const uint16_t* palette, const uint16_t* bias,
                           int n, int epi, const uint16_t* residual, const float* rope,
                           int rope_rows, uint16_t* y, const int32_t* rope_pos = nullptr);
sam3_status_t gemm_dense(sam3_ctx_t* ctx, const uint16_t* x, int m, int k, const uint16_t* w,
                         const uint16_t* bias, int n, uint16_t* y,
                         int prof_class = SAM3_PROF_PATCH);
sam3_status_t layernorm(sam3_ctx_t* ctx, const uint16_t* x, int m, int d, const uint16_t* g,
                        const uint16_t* b, float eps, uint16_t* y);
sam3_status_t attention(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                        int head_dim, float scale, uint16_t* o);
// Attention over `groups` row groups of `seq` rows per image: group g of image
// i is rows i*img_rows + first_row + g*seq ... (windowed attention).
sam3_status_t attention_grouped(sam3_ctx_t* ctx, const uint16_t* qkv, int images, int groups,
                                int seq, int img_rows, int first_row, int heads, int head_dim,
                                float scale, uint16_t* o);
sam3_status_t rope_table(sam3_ctx_t* ctx, int gh, int gw, int hd, float theta, float* t);
// Once per context: the grid table (ctx->rope), its axial form and the
// grid-order row coordinates for max_batch images.
sam3_status_t rope_setup(sam3_ctx_t* ctx);
// out[i] = coordinates x | y << 16 of grid token idx[i] (grid width gw).
sam3_status_t rope_pos_from_idx(sam3_ctx_t* ctx, const int32_t* idx, int n, int gw, int32_t* out);
sam3_status_t prune(sam3_ctx_t* ctx, const uint16_t* x, int batch, int seq, int d, int keep,
                    int norm, int order, const float* rope_in, int rope_rows, int rope_cols,
                    uint16_t* feats, float* rope_out, int32_t* idx, float* scores_scratch);
// image: fp16 RGB NHWC, or f32 RGBA NHWC in [0, 1] normalised on the fly
// (rgba = true).
sam3_status_t patch_embed(sam3_ctx_t* ctx, const void* image, bool rgba, int batch, int h, int w,
                          const uint16_t* pw, const uint16_t* pb, int patch, int dim,
                          uint16_t* out, uint16_t* cols_scratch, uint16_t* wpad_scratch);

// Launch with programmatic stream serialization: the kernel may start while
// the previous kernel in the stream finishes (its prologue overlapping that
// kernel's tail) and must call griddep_wait before touching that kernel's
// outputs (or any buffer a preceding kernel reads or writes).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// A plain launch (no attributes) that returns its own error instead of
// leaving it only in the thread's last-error state.
template <typename... KArgs, typename... Args>
cudaError_t launch_plain(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Brackets one launch with CUDA events when the context is profiling.
class ProfScope {
 public:
  ProfScope(sam3_ctx_t* ctx, int cls, double flops, double bytes);
  ~ProfScope();

 private:
  sam3_ctx_t* ctx_;
  int idx_ = -1;
};

}  // namespace sam3

#define SAM3_CHECK_CTX(ctx) \
  do {                      \
    if (!(ctx)) return SAM3_ERR_INVALID_ARG; \
  } while (0)
