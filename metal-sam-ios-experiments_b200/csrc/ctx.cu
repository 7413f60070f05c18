// ctx.cu - context, workspace arena, memory helpers and error reporting.
//
// Replaces the reference's process-global CompiledGraphCache / BufferAllocator
// (OptimizationInfrastructure.swift:20-332): instead of a locked size-bucket
// pool, each context owns one arena sized for cfg.max_batch images, carved
// once at creation, so the encoder's hot loop never allocates.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace sam3 {

sam3_status_t set_error(sam3_ctx_t* ctx, sam3_status_t code, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return code;
}

sam3_status_t check_cuda(sam3_ctx_t* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SAM3_OK;
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return set_error(ctx, SAM3_ERR_OOM, "%s: %s", what, cudaGetErrorString(e));
  }
  return set_error(ctx, SAM3_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

sam3_status_t check_launch(sam3_ctx_t* ctx, const char* what) {
  ctx->launches++;
  sam3_status_t st = check_cuda(ctx, cudaGetLastError(), what);
  if (st == SAM3_OK && (ctx->fault & SAM3_FAULT_LAUNCH))
    return set_error(ctx, SAM3_ERR_CUDA, "%s: injected launch failure", what);
  return st;
}

sam3_status_t check_launch_ret(sam3_ctx_t* ctx, cudaError_t e, const char* what) {
  const cudaError_t last = cudaGetLastError();  // clears a launch error recorded twice
  ctx->launches++;
  sam3_status_t st = check_cuda(ctx, e != cudaSuccess ? e : last, what);
  if (st == SAM3_OK && (ctx->fault & SAM3_FAULT_LAUNCH))
    return set_error(ctx, SAM3_ERR_CUDA, "%s: injected launch failure", what);
  return st;
}

namespace {

// One thread waits, with the bounded wait every kernel uses, on an mbarrier
// that nothing arrives on: the wait runs out after kWaitTimeoutNs, records
// kDevErrTimeoutSelftest in the context's error word and the kernel returns.
__global__ void selftest_wait_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, err, kDevErrTimeoutSelftest);
}

int fault_flags_from_env() {
  const char* v = getenv("SAM3_FAULT");
  int f = 0;
  if (v) {
    if (strstr(v, "alloc")) f |= SAM3_FAULT_ALLOC;
    if (strstr(v, "launch")) f |= SAM3_FAULT_LAUNCH;
  }
  return f;
}

}  // namespace

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

ProfScope::ProfScope(sam3_ctx_t* ctx, int cls, double flops, double bytes) : ctx_(ctx) {
  if (!ctx->profiling) return;
  cudaEvent_t ev[2];
  for (int i = 0; i < 2; ++i) {
    if (!ctx->event_pool.empty()) {
      ev[i] = ctx->event_pool.back();
      ctx->event_pool.pop_back();
    } else if (cudaEventCreate(&ev[i]) != cudaSuccess) {
      cudaGetLastError();
      if (i == 1) ctx->event_pool.push_back(ev[0]);
      return;
    }
  }
  cudaEventRecord(ev[0], ctx->stream);
  ctx->prof_pending.push_back({cls, flops, bytes, ev[0], ev[1]});
  idx_ = (int)ctx->prof_pending.size() - 1;
}

ProfScope::~ProfScope() {
  if (idx_ >= 0) cudaEventRecord(ctx_->prof_pending[(size_t)idx_].stop, ctx_->stream);
}

namespace {

void resolve_profile(sam3_ctx_t* ctx) {
  cudaStreamSynchronize(ctx->stream);
  for (auto& r : ctx->prof_pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, r.start, r.stop) == cudaSuccess) {
      ctx->prof.launches[r.cls] += 1;
      ctx->prof.milliseconds[r.cls] += ms;
      ctx->prof.flops[r.cls] += r.flops;
      ctx->prof.bytes[r.cls] += r.bytes;
    } else {
      cudaGetLastError();
    }
    ctx->event_pool.push_back(r.start);
    ctx->event_pool.push_back(r.stop);
  }
  ctx->prof_pending.clear();
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Carver {
  char* base;
  size_t off = 0;
  template <class T>
  T* take(size_t count) {
    off = align_up(off, 256);
    T* p = reinterpret_cast<T*>(base + off);
    off += count * sizeof(T);
    return p;
  }
};

// Lay out (or, with base == nullptr, just measure) the encoder workspace.
size_t carve(sam3_ctx_t* ctx, char* base) {
  const sam3_encoder_config_t& c = ctx->cfg;
  const size_t B = (size_t)std::max(1, c.max_batch);
  const size_t grid = (size_t)(c.image_size / c.patch);
  const size_t S = grid * grid;
  const size_t D = (size_t)c.embed_dim, F = (size_t)c.mlp_hidden;
  const size_t keep = (size_t)std::min<int64_t>(c.keep_tokens, (int64_t)S);
  const size_t hd = D / (size_t)c.num_heads;
  const size_t kp = align_up(3u * c.patch * c.patch, 64);
  // activation rows per image: the S patch tokens plus one class token
  // (the windowed encoder variant); the plain encoder uses the first S
  const size_t R = S + 1;
  Carver cv{base};
  ctx->x = cv.take<uint16_t>(B * R * D);
  ctx->xp = cv.take<uint16_t>(B * keep * D);
  ctx->ln = cv.take<uint16_t>(B * R * D);
  ctx->qkv = cv.take<uint16_t>(B * R * 3 * D);
  ctx->attn = cv.take<uint16_t>(B * R * D);
  ctx->hidden = cv.take<uint16_t>(B * R * F);
  ctx->cols = cv.take<uint16_t>(B * S * kp);
  ctx->patch_wp = cv.take<uint16_t>(D * kp);
  ctx->scores = cv.take<float>(B * S);
  ctx->rope = cv.take<float>(S * hd);
  ctx->rope_axial = cv.take<float>(grid * 32);
  ctx->rope_pos_grid = cv.take<int32_t>(B * S);
  ctx->rope_pos_win = cv.take<int32_t>(B * R);
  ctx->rope_pos_pruned = cv.take<int32_t>(B * keep);
  ctx->rope_pruned = cv.take<float>(B * keep * hd);
  ctx->idx = cv.take<int32_t>(B * S);
  ctx->image = cv.take<uint16_t>(B * (size_t)c.image_size * c.image_size * 3);
  ctx->block_rows = B * S;
  ctx->token_rows = B * R;
  return align_up(cv.off, 256);
}

}  // namespace

sam3_status_t ensure_workspace(sam3_ctx_t* ctx) {
  const size_t need = carve(ctx, nullptr);
  if (ctx->ws && ctx->ws_bytes >= need) {
    carve(ctx, ctx->ws);
    return SAM3_OK;
  }
  if (ctx->ws) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  void* p = nullptr;
  sam3_status_t st = check_cuda(ctx, cudaMalloc(&p, need), "workspace cudaMalloc");
  if (st != SAM3_OK) return st;
  ctx->ws = static_cast<char*>(p);
  ctx->ws_bytes = need;
  ctx->rope_ready = 0;
  ctx->rope_win_key = 0;
  carve(ctx, ctx->ws);
  return SAM3_OK;
}

sam3_status_t device_error_status(sam3_ctx_t* ctx, int err) {
  if (!err) return SAM3_OK;
  if ((err & 0xF00) == 0x200)  // a kernel met an invalid index in its input and skipped it
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "index out of range in a kernel input (code 0x%x)",
                     err);
  return set_error(ctx, SAM3_ERR_TIMEOUT, "kernel bounded wait expired (code 0x%x)", err);
}

}  // namespace sam3

using namespace sam3;

extern "C" {

sam3_status_t sam3_config_default(sam3_encoder_config_t* c) {
  if (!c) return SAM3_ERR_INVALID_ARG;
  c->embed_dim = 1024;
  c->num_heads = 16;
  c->mlp_hidden = 4096;
  c->num_blocks = 32;
  c->patch = 14;
  c->image_size = 1008;
  c->prune_after_block = 16;
  c->keep_tokens = 2592;
  c->score_norm = SAM3_SCORE_L2;
  c->keep_order = SAM3_ORDER_INDEX;
  c->ln_eps = 1e-6f;
  c->rope_theta = 10000.0f;
  c->max_batch = 1;
  return SAM3_OK;
}

static sam3_status_t validate_config(const sam3_encoder_config_t& c) {
  if (c.embed_dim <= 0 || c.num_heads <= 0 || c.embed_dim % c.num_heads) return SAM3_ERR_SHAPE;
  if (c.embed_dim / c.num_heads != 64) return SAM3_ERR_SHAPE;
  if (c.embed_dim % 128 || c.mlp_hidden % 128 || c.mlp_hidden <= 0) return SAM3_ERR_SHAPE;
  if (c.patch <= 0 || c.image_size <= 0 || c.image_size % c.patch) return SAM3_ERR_SHAPE;
  if (c.num_blocks < 0 || c.prune_after_block < 0 || c.keep_tokens <= 0) return SAM3_ERR_SHAPE;
  const int grid = c.image_size / c.patch;
  if ((int64_t)grid * grid > 16384) return SAM3_ERR_SHAPE;
  if (c.score_norm != SAM3_SCORE_L2 && c.score_norm != SAM3_SCORE_L1) return SAM3_ERR_INVALID_ARG;
  if (c.keep_order != SAM3_ORDER_INDEX && c.keep_order != SAM3_ORDER_SCORE)
    return SAM3_ERR_INVALID_ARG;
  if (c.max_batch <= 0 || c.max_batch > 64) return SAM3_ERR_SHAPE;
  return SAM3_OK;
}

sam3_status_t sam3_ctx_create(int device, const sam3_encoder_config_t* cfg, sam3_ctx_t** out) {
  if (!out) return SAM3_ERR_INVALID_ARG;
  *out = nullptr;
  sam3_encoder_config_t c;
  if (cfg)
    c = *cfg;
  else
    sam3_config_default(&c);
  sam3_status_t st = validate_config(c);
  if (st != SAM3_OK) return st;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return SAM3_ERR_UNSUPPORTED;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return SAM3_ERR_CUDA;
  if (prop.major != 10 || prop.minor != 0) return SAM3_ERR_UNSUPPORTED;  // sm_100 only
  if (cudaSetDevice(device) != cudaSuccess) return SAM3_ERR_CUDA;
  if (!encode_tiled()) return SAM3_ERR_UNSUPPORTED;

  sam3_ctx_t* ctx = new sam3_ctx_t();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->cfg = c;
  if ((st = check_cuda(ctx, cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking),
                       "cudaStreamCreate")) != SAM3_OK) {
    delete ctx;
    return st;
  }
  ctx->stream = ctx->own_stream;
  if ((st = check_cuda(ctx, cudaMalloc(&ctx->dev_err, sizeof(int)), "cudaMalloc err")) !=
      SAM3_OK) {
    sam3_ctx_destroy(ctx);
    return st;
  }
  cudaMemset(ctx->dev_err, 0, sizeof(int));
  if ((st = ensure_workspace(ctx)) != SAM3_OK) {
    sam3_ctx_destroy(ctx);
    return st;
  }
  cudaDeviceSynchronize();
  ctx->fault = fault_flags_from_env();  // after the workspace: the context itself is made
  *out = ctx;
  return SAM3_OK;
}

sam3_status_t sam3_set_fault(sam3_ctx_t* ctx, int32_t flags) {
  SAM3_CHECK_CTX(ctx);
  if (flags & ~(SAM3_FAULT_ALLOC | SAM3_FAULT_LAUNCH)) return SAM3_ERR_INVALID_ARG;
  ctx->fault = flags;
  return SAM3_OK;
}

int32_t sam3_get_fault(const sam3_ctx_t* ctx) { return ctx ? ctx->fault : 0; }

sam3_status_t sam3_selftest_wait_timeout(sam3_ctx_t* ctx) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  selftest_wait_kernel<<<1, 32, 0, ctx->stream>>>(ctx->dev_err);
  return check_launch(ctx, "selftest_wait_kernel");
}

sam3_status_t sam3_ctx_destroy(sam3_ctx_t* ctx) {
  if (!ctx) return SAM3_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  resolve_profile(ctx);
  for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
  if (ctx->copy_stream) cudaStreamSynchronize(ctx->copy_stream);
  if (ctx->down_stream) cudaStreamSynchronize(ctx->down_stream);
  for (cudaEvent_t e : ctx->pipe_ev)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : ctx->pipe_done)
    if (e) cudaEventDestroy(e);
  if (ctx->pipe_err) cudaFreeHost(ctx->pipe_err);
  if (ctx->pipe_mem) cudaFree(ctx->pipe_mem);
  if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
  if (ctx->down_stream) cudaStreamDestroy(ctx->down_stream);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->dev_err) cudaFree(ctx->dev_err);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return SAM3_OK;
}

sam3_status_t sam3_ctx_set_stream(sam3_ctx_t* ctx, void* s) {
  SAM3_CHECK_CTX(ctx);
  ctx->stream = s ? static_cast<cudaStream_t>(s) : ctx->own_stream;
  return SAM3_OK;
}

void* sam3_ctx_stream(sam3_ctx_t* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

const char* sam3_last_error(const sam3_ctx_t* ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

uint64_t sam3_launch_count(const sam3_ctx_t* ctx) { return ctx ? ctx->launches : 0; }

sam3_status_t sam3_sync(sam3_ctx_t* ctx) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  sam3_status_t st = check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "stream sync");
  if (st != SAM3_OK) return st;
  int err = 0;
  st = check_cuda(ctx, cudaMemcpy(&err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost),
                  "read device error word");
  if (st != SAM3_OK) return st;
  if (err) cudaMemset(ctx->dev_err, 0, sizeof(int));
  return sam3::device_error_status(ctx, err);
}

sam3_status_t sam3_profile_enable(sam3_ctx_t* ctx, int32_t enable) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  resolve_profile(ctx);
  ctx->prof = sam3_profile_t{};
  ctx->profiling = enable != 0;
  return SAM3_OK;
}

sam3_status_t sam3_profile_read(sam3_ctx_t* ctx, sam3_profile_t* out) {
  SAM3_CHECK_CTX(ctx);
  if (!out) return SAM3_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  resolve_profile(ctx);
  *out = ctx->prof;
  return SAM3_OK;
}

sam3_status_t sam3_alloc(sam3_ctx_t* ctx, size_t bytes, void** p) {
  SAM3_CHECK_CTX(ctx);
  if (!p) return SAM3_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  if (ctx->fault & SAM3_FAULT_ALLOC) {
    *p = nullptr;
    return set_error(ctx, SAM3_ERR_OOM, "sam3_alloc: injected allocation failure");
  }
  return check_cuda(ctx, cudaMalloc(p, bytes ? bytes : 1), "sam3_alloc");
}
sam3_status_t sam3_free(sam3_ctx_t* ctx, void* p) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  return check_cuda(ctx, cudaFree(p), "sam3_free");
}
sam3_status_t sam3_host_alloc(sam3_ctx_t* ctx, size_t bytes, void** p) {
  SAM3_CHECK_CTX(ctx);
  if (!p) return SAM3_ERR_INVALID_ARG;
  if (ctx->fault & SAM3_FAULT_ALLOC) {
    *p = nullptr;
    return set_error(ctx, SAM3_ERR_OOM, "sam3_host_alloc: injected allocation failure");
  }
  return check_cuda(ctx, cudaMallocHost(p, bytes ? bytes : 1), "sam3_host_alloc");
}
sam3_status_t sam3_host_free(sam3_ctx_t* ctx, void* p) {
  SAM3_CHECK_CTX(ctx);
  return check_cuda(ctx, cudaFreeHost(p), "sam3_host_free");
}
sam3_status_t sam3_upload(sam3_ctx_t* ctx, void* dst, const void* src, size_t bytes) {
  SAM3_CHECK_CTX(ctx);
  if (!dst || !src) return SAM3_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  sam3_status_t st = check_cuda(
      ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "upload");
  if (st != SAM3_OK) return st;
  return check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "upload sync");
}
sam3_status_t sam3_download(sam3_ctx_t* ctx, void* dst, const void* src, size_t bytes) {
  SAM3_CHECK_CTX(ctx);
  if (!dst || !src) return SAM3_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  sam3_status_t st = check_cuda(
      ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "download");
  if (st != SAM3_OK) return st;
  return check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "download sync");
}

}  // extern "C"
