// small_ops.cu - the HBM-bound operators of the path: LayerNorm, the RoPE
// table and stand-alone RoPE, token scores, token pruning (radix select +
// stable compaction + gather) and the patch-embedding im2col.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace sam3 {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row; lane owns 8-element chunks lane*8 + j*256 (coalesced
// 512-byte warp accesses). Two-pass mean/variance in fp32 registers.
// Reference: LayerNorm.forward, ViTEncoder.swift:795-887 (graph.normalize
// with biased variance, epsilon 1e-6).
template <int NCH>
__global__ void __launch_bounds__(256) layernorm_kernel(const __half* __restrict__ x, int m,
                                                        const __half* __restrict__ g,
                                                        const __half* __restrict__ b, float eps,
                                                        __half* __restrict__ y) {
  constexpr int D = NCH * 256;
  griddep_launch_dependents();
  griddep_wait();  // x is the previous kernel's output
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * D);
  float v[NCH][8];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const uint4 u = __ldg(xr + lane + 32 * j);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 p = unpack_half2(w[q]);
      v[j][2 * q] = p.x;
      v[j][2 * q + 1] = p.y;
      s += p.x + p.y;
    }
  }
  const float mean = warp_sum(s) * (1.0f / D);
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < NCH; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float t = v[j][e] - mean;
      var += t * t;
    }
  const float rstd = 1.0f / sqrtf(warp_sum(var) * (1.0f / D) + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * D);
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int c0 = (lane + 32 * j) * 8;
    float gg[8], bb[8];
    if (g) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(g + c0));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 p = unpack_half2(w[q]);
        gg[2 * q] = p.x;
        gg[2 * q + 1] = p.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) gg[e] = 1.f;
    }
    if (b) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(b + c0));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 p = unpack_half2(w[q]);
        bb[2 * q] = p.x;
        bb[2 * q + 1] = p.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) bb[e] = 0.f;
    }
    uint4 o;
    uint32_t* ow = &o.x;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      ow[q] = pack_half2((v[j][2 * q] - mean) * rstd * gg[2 * q] + bb[2 * q],
                         (v[j][2 * q + 1] - mean) * rstd * gg[2 * q + 1] + bb[2 * q + 1]);
    yr[lane + 32 * j] = o;
  }
}

// ---------------------------------------------------------------- RoPE
// Reference: compute_rope_freqs_2d, Metal/RoPE.metal:22-52.
__global__ void rope_table_kernel(float* __restrict__ t, int gh, int gw, int hd, float theta) {
  const int quarter = hd / 4;
  const int p = blockIdx.x * blockDim.y + threadIdx.y;
  const int i = threadIdx.x;
  if (p >= gh * gw || i >= quarter) return;
  const int h = p / gw, w = p % gw;
  const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)(2 * quarter));
  const float ax = (float)w * freq, ay = (float)h * freq;
  float2* row = reinterpret_cast<float2*>(t + (size_t)p * hd);
  row[i] = make_float2(cosf(ax), sinf(ax));
  row[quarter + i] = make_float2(cosf(ay), sinf(ay));
}

// Axial form of the table, pair-major: pair i (i < 16) at coordinate c is
// float2 element ((i / 2) * coords + c) * 2 + i % 2, i.e. the float4 of pairs
// (2q, 2q+1) of all coordinates are contiguous (consecutive tokens of a warp
// read consecutive entries in the QKV epilogue). The row-index half of the
// table uses the same frequencies and formula as the column-index half, so
// row c (h = 0, w = c) gives coordinate c for both halves bit for bit; rows
// h*gw (w = 0) cover c >= gw on taller grids.
__global__ void rope_axial_kernel(const float2* __restrict__ t, int gw, int coords,
                                  float2* __restrict__ a) {
  const int c = blockIdx.x, i = threadIdx.x;
  a[((i >> 1) * coords + c) * 2 + (i & 1)] =
      c < gw ? t[(size_t)c * 32 + i] : t[(size_t)c * gw * 32 + 16 + i];
}

// pos[r] = coordinates of grid token r % per, x | y << 16.
__global__ void rope_pos_grid_kernel(int32_t* __restrict__ pos, int rows, int per, int gw) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int p = r % per;
  pos[r] = (p % gw) | ((p / gw) << 16);
}

__global__ void rope_pos_idx_kernel(const int32_t* __restrict__ idx, int n, int gw,
                                    int32_t* __restrict__ pos) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int p = idx[i];
  pos[i] = (p % gw) | ((p / gw) << 16);
}

// Reference: apply_rope_2d_batch, Metal/RoPE.metal:111-153 (packed QKV row,
// q and k rotated, v untouched).
__global__ void rope_apply_kernel(__half2* __restrict__ qkv, int m, int dim, int hd,
                                  const float2* __restrict__ t, int rows) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)m * dim) return;
  const int row = (int)(i / dim), pr = (int)(i % dim);
  const int col = 2 * pr;  // column inside the q|k region
  const int j = (col % hd) / 2;
  const float2 cs = t[(size_t)(row % rows) * (hd / 2) + j];
  __half2* p = qkv + ((size_t)row * 3 * dim + col) / 2;
  const float2 v = __half22float2(*p);
  *p = __floats2half2_rn(v.x * cs.x - v.y * cs.y, v.x * cs.y + v.y * cs.x);
}

// ---------------------------------------------------------------- pruning
// Score per token. Reference: TokenPruner.swift:54-56 (L1 = sum |x|); the
// benchmark spec uses the L2 norm.
__global__ void __launch_bounds__(256) token_score_kernel(const __half* __restrict__ x, int rows,
                                                          int d, int norm,
                                                          float* __restrict__ scores) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * d);
  float s = 0.f;
  for (int c = lane; c < d / 8; c += 32) {
    const uint4 u = __ldg(xr + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 p = unpack_half2(w[q]);
      s += norm == SAM3_SCORE_L1 ? fabsf(p.x) + fabsf(p.y) : p.x * p.x + p.y * p.y;
    }
  }
  s = warp_sum(s);
  if (lane == 0) scores[row] = norm == SAM3_SCORE_L1 ? s : sqrtf(s);
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Block-wide exclusive scan of per-thread counts (1024 threads).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    warp_sums[lane] = wi - w;
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const int r = warp_sums[warp] + inc - v;
  __syncthreads();
  return r;
}

// One CTA (1024 threads) per image: 4 passes of 8-bit radix selection find
// the keep-th largest score key T and how many ties at T to take; ties go to
// the lower token index; a stable compaction emits the kept indices in
// ascending order, or a bitonic sort orders them by (score desc, index asc).
// Reference: the topK of TokenPruner.swift:59-60 (MPSGraph, ties undefined).
__global__ void __launch_bounds__(1024) prune_select_kernel(const float* __restrict__ scores,
                                                            int seq, int keep, int order,
                                                            int32_t* __restrict__ idx_out) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm);
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ int s_total;
  __shared__ uint32_t s_prefix;
  __shared__ int s_needed;
  const int b = blockIdx.x;
  const float* sc = scores + (size_t)b * seq;
  for (int i = threadIdx.x; i < seq; i += blockDim.x) keys[i] = order_key(sc[i]);
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_needed = keep;
  }
  __syncthreads();
  uint32_t mask = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = threadIdx.x; i < seq; i += blockDim.x)
      if ((keys[i] & mask) == prefix) atomicAdd(&hist[(keys[i] >> shift) & 255u], 1);
    __syncthreads();
    if (threadIdx.x == 0) {
      int cum = 0, need = s_needed;
      for (int dgt = 255; dgt >= 0; --dgt) {
        if (cum + hist[dgt] >= need) {
          s_prefix = prefix | ((uint32_t)dgt << shift);
          s_needed = need - cum;
          break;
        }
        cum += hist[dgt];
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const int ties = s_needed;  // how many tokens with key == T to keep

  // Contiguous chunk per thread keeps index order inside the scans.
  const int per = (seq + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(seq, lo + per);
  int n_eq = 0;
  for (int i = lo; i < hi; ++i) n_eq += keys[i] == T;
  const int eq0 = block_exclusive_scan(n_eq, warp_sums, &s_total);  // ties before my chunk
  int eq_rank = eq0, n_sel = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t k = keys[i];
    if (k > T) ++n_sel;
    else if (k == T) n_sel += (eq_rank++ < ties);
  }
  int pos = block_exclusive_scan(n_sel, warp_sums, &s_total);
  eq_rank = eq0;
  int32_t* out = idx_out + (size_t)b * keep;
  if (order == SAM3_ORDER_INDEX) {
    for (int i = lo; i < hi; ++i) {
      const uint32_t k = keys[i];
      bool take = k > T;
      if (k == T) take = eq_rank++ < ties;
      if (take) out[pos++] = i;
    }
    return;
  }
  // SAM3_ORDER_SCORE: bitonic sort of (~key << 32 | index) ascending.
  int p2 = 1;
  while (p2 < keep) p2 <<= 1;
  unsigned long long* sk = reinterpret_cast<unsigned long long*>(sm + (((size_t)seq * 4 + 15) & ~15));
  for (int i = threadIdx.x; i < p2; i += blockDim.x) sk[i] = ~0ull;
  __syncthreads();
  for (int i = lo; i < hi; ++i) {
    const uint32_t k = keys[i];
    bool take = k > T;
    if (k == T) take = eq_rank++ < ties;
    if (take) sk[pos++] = ((unsigned long long)(~k) << 32) | (uint32_t)i;
  }
  __syncthreads();
  for (int size = 2; size <= p2; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < p2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = sk[i], c = sk[j];
          if ((a > c) == up) {
            sk[i] = c;
            sk[j] = a;
          }
        }
      }
      __syncthreads();
    }
  for (int i = threadIdx.x; i < keep; i += blockDim.x) out[i] = (int32_t)(sk[i] & 0xffffffffu);
}

// Gather kept rows (features fp16, RoPE rows f32). One warp per output row.
__global__ void __launch_bounds__(256) prune_gather_kernel(
    const __half* __restrict__ x, int seq, int d, int keep, const int32_t* __restrict__ idx,
    const float* __restrict__ rope_in, int rope_rows, int rope_cols, __half* __restrict__ feats,
    float* __restrict__ rope_out, int total) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= total) return;
  const int b = r / keep;
  const long long src = (long long)b * seq + idx[r];
  const uint4* s = reinterpret_cast<const uint4*>(x + src * d);
  uint4* dst = reinterpret_cast<uint4*>(feats + (size_t)r * d);
  for (int c = lane; c < d / 8; c += 32) dst[c] = __ldg(s + c);
  if (rope_in && rope_out) {
    const float* rs = rope_in + (size_t)(src % rope_rows) * rope_cols;
    float* rd = rope_out + (size_t)r * rope_cols;
    for (int c = lane; c < rope_cols; c += 32) rd[c] = __ldg(rs + c);
  }
}

// ---------------------------------------------------------------- patch embedding
// im2col of an NHWC fp16 image into [tokens, kp] rows (k = c*P*P + ky*P + kx,
// the PyTorch conv-weight order), zero-padded from 3*P*P up to kp.
// ImageNet statistics the reference normalises camera frames with
// (SAM3Predictor.swift:334-335).
__constant__ float kImageMean[3] = {0.485f, 0.456f, 0.406f};
__constant__ float kImageStd[3] = {0.229f, 0.224f, 0.225f};

// (x - mean[c]) / std[c] in fp32 (IEEE division), rounded to fp16: the
// reference's slice_rgb -> sub_mean -> div_std (SAM3Predictor.swift:332-341).
__device__ __forceinline__ __half normalize_channel(float x, int c) {
  return __float2half_rn(__fdiv_rn(x - kImageMean[c], kImageStd[c]));
}

// One CTA per token: its patch is written as the GEMM A row [c][ky][kx]
// (the conv weight order), zero-padded to kp columns. RGBA: the image is f32
// RGBA [B, H, W, 4] in [0, 1] and is normalised on the fly (the A-operand side
// of the reference's preprocessing); otherwise fp16 RGB [B, H, W, 3].
template <bool RGBA>
__global__ void __launch_bounds__(128) im2col_kernel(const void* __restrict__ img, int h, int w,
                                                     int patch, int kp, __half* __restrict__ cols) {
  const int gw = w / patch, gh = h / patch;
  const int token = blockIdx.x;
  const int b = token / (gh * gw), p = token - b * (gh * gw);
  const int y0 = (p / gw) * patch, x0 = (p - (p / gw) * gw) * patch;
  const int pp = patch * patch;
  __half* out = cols + (size_t)token * kp;
  for (int k = threadIdx.x; k < kp; k += blockDim.x) {
    __half v = __float2half_rn(0.f);
    if (k < 3 * pp) {
      const int c = k / pp, r = k - c * pp, ky = r / patch, kx = r - ky * patch;
      const size_t pix = ((size_t)b * h + y0 + ky) * w + x0 + kx;
      if (RGBA)
        v = normalize_channel(__ldg(static_cast<const float*>(img) + pix * 4 + c), c);
      else
        v = static_cast<const __half*>(img)[pix * 3 + c];
    }
    out[k] = v;
  }
}

// Stand-alone preprocessing: f32 RGBA [pixels, 4] -> fp16 RGB [pixels, 3].
__global__ void preprocess_rgba_kernel(const float4* __restrict__ rgba, long long pixels,
                                       __half* __restrict__ rgb) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < pixels;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = __ldg(rgba + i);
    rgb[3 * i] = normalize_channel(v.x, 0);
    rgb[3 * i + 1] = normalize_channel(v.y, 1);
    rgb[3 * i + 2] = normalize_channel(v.z, 2);
  }
}

__global__ void pad_weight_kernel(const __half* __restrict__ w, int n, int k, int kp,
                                  __half* __restrict__ wp) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)n * kp) return;
  const int c = (int)(i % kp);
  const long long r = i / kp;
  wp[i] = c < k ? w[r * k + c] : __float2half(0.f);
}

int blocks_for(long long n, int t) { return (int)((n + t - 1) / t); }

}  // namespace

sam3_status_t layernorm(sam3_ctx_t* ctx, const uint16_t* x, int m, int d, const uint16_t* g,
                        const uint16_t* b, float eps, uint16_t* y) {
  if (!x || !y) return set_error(ctx, SAM3_ERR_INVALID_ARG, "layernorm: null pointer");
  if (m <= 0 || d <= 0) return set_error(ctx, SAM3_ERR_SHAPE, "layernorm: empty shape");
  if (!aligned16(x) || !aligned16(y) || (g && !aligned16(g)) || (b && !aligned16(b)))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "layernorm: pointers must be 16-byte aligned");
  const __half* hx = reinterpret_cast<const __half*>(x);
  const __half* hg = reinterpret_cast<const __half*>(g);
  const __half* hb = reinterpret_cast<const __half*>(b);
  __half* hy = reinterpret_cast<__half*>(y);
  const int grid = blocks_for(m, 8);
  ProfScope prof(ctx, SAM3_PROF_LAYERNORM, 0.0, 4.0 * m * d);
  void (*kern)(const __half*, int, const __half*, const __half*, float, __half*) = nullptr;
  switch (d) {
    case 256: kern = layernorm_kernel<1>; break;
    case 512: kern = layernorm_kernel<2>; break;
    case 768: kern = layernorm_kernel<3>; break;
    case 1024: kern = layernorm_kernel<4>; break;
    case 1280: kern = layernorm_kernel<5>; break;
    case 1536: kern = layernorm_kernel<6>; break;
    case 2048: kern = layernorm_kernel<8>; break;
    default:
      return set_error(ctx, SAM3_ERR_SHAPE, "layernorm: d=%d unsupported (256..2048, step 256)", d);
  }
  return check_launch_ret(ctx, launch_pdl(kern, dim3(grid), dim3(256), 0, ctx->stream, hx, m, hg,
                                          hb, eps, hy),
                          "layernorm_kernel");
}

sam3_status_t rope_table(sam3_ctx_t* ctx, int gh, int gw, int hd, float theta, float* t) {
  if (!t) return set_error(ctx, SAM3_ERR_INVALID_ARG, "rope_table: null table");
  if (gh <= 0 || gw <= 0 || hd <= 0 || hd % 4 || hd > 256)
    return set_error(ctx, SAM3_ERR_SHAPE, "rope_table: bad grid/head_dim");
  const int quarter = hd / 4;
  const int per = std::max(1, 256 / quarter);
  ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 4.0 * gh * gw * hd);
  rope_table_kernel<<<blocks_for((long long)gh * gw, per), dim3(quarter, per), 0, ctx->stream>>>(
      t, gh, gw, hd, theta);
  return check_launch(ctx, "rope_table_kernel");
}

sam3_status_t rope_setup(sam3_ctx_t* ctx) {
  if (ctx->rope_ready) return SAM3_OK;
  const sam3_encoder_config_t& c = ctx->cfg;
  const int grid = c.image_size / c.patch, S = grid * grid;
  const int hd = c.embed_dim / c.num_heads;
  sam3_status_t st = rope_table(ctx, grid, grid, hd, c.rope_theta, ctx->rope);
  if (st != SAM3_OK) return st;
  if (hd == 64) {  // the axial form serves the QKV epilogue (head_dim 64)
    ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 2.0 * grid * 16 * 8);
    rope_axial_kernel<<<grid, 16, 0, ctx->stream>>>(reinterpret_cast<const float2*>(ctx->rope),
                                                     grid, grid,
                                                     reinterpret_cast<float2*>(ctx->rope_axial));
    if ((st = check_launch(ctx, "rope_axial_kernel")) != SAM3_OK) return st;
    const int rows = std::max(1, c.max_batch) * S;
    rope_pos_grid_kernel<<<blocks_for(rows, 256), 256, 0, ctx->stream>>>(ctx->rope_pos_grid, rows,
                                                                         S, grid);
    if ((st = check_launch(ctx, "rope_pos_grid_kernel")) != SAM3_OK) return st;
  }
  ctx->rope_ready = 1;
  return SAM3_OK;
}

sam3_status_t rope_pos_from_idx(sam3_ctx_t* ctx, const int32_t* idx, int n, int gw, int32_t* out) {
  if (n <= 0) return SAM3_OK;
  ProfScope prof(ctx, SAM3_PROF_PRUNE, 0.0, 8.0 * n);
  rope_pos_idx_kernel<<<blocks_for(n, 256), 256, 0, ctx->stream>>>(idx, n, gw, out);
  return check_launch(ctx, "rope_pos_idx_kernel");
}

// prune_select_kernel's largest dynamic shared memory: seq <= 16384 score
// keys plus, in score order, a bitonic buffer of up to 8192 (key, index) pairs.
constexpr int kPruneSelectSmemMax = 16384 * 4 + 8192 * 8;

sam3_status_t prune(sam3_ctx_t* ctx, const uint16_t* x, int batch, int seq, int d, int keep,
                    int norm, int order, const float* rope_in, int rope_rows, int rope_cols,
                    uint16_t* feats, float* rope_out, int32_t* idx, float* scores) {
  if (!x || !feats || !idx || !scores)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "prune: null pointer");
  if (batch <= 0 || seq <= 0 || d <= 0 || d % 8 || keep <= 0 || keep > seq || seq > 16384)
    return set_error(ctx, SAM3_ERR_SHAPE, "prune: bad shape batch=%d seq=%d d=%d keep=%d", batch,
                     seq, d, keep);
  if (norm != SAM3_SCORE_L2 && norm != SAM3_SCORE_L1)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "prune: bad norm");
  if (order != SAM3_ORDER_INDEX && order != SAM3_ORDER_SCORE)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "prune: bad order");
  if (order == SAM3_ORDER_SCORE && keep > 8192)
    return set_error(ctx, SAM3_ERR_SHAPE, "prune: score order supports keep <= 8192");
  if ((rope_in == nullptr) != (rope_out == nullptr) || (rope_in && (rope_rows <= 0 || rope_cols <= 0)))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "prune: rope_in/rope_out mismatch");
  if (!aligned16(x) || !aligned16(feats))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "prune: x/feats must be 16-byte aligned");
  const long long rows = (long long)batch * seq;
  sam3_status_t st;
  {
    ProfScope prof(ctx, SAM3_PROF_PRUNE, 0.0, 2.0 * rows * d + 4.0 * rows);
    token_score_kernel<<<blocks_for(rows, 8), 256, 0, ctx->stream>>>(
        reinterpret_cast<const __half*>(x), (int)rows, d, norm, scores);
    st = check_launch(ctx, "token_score_kernel");
  }
  if (st != SAM3_OK) return st;
  size_t smem = ((size_t)seq * 4 + 15) & ~(size_t)15;
  if (order == SAM3_ORDER_SCORE) {
    int p2 = 1;
    while (p2 < keep) p2 <<= 1;
    smem += (size_t)p2 * 8;
  }
  // The limit is raised once per device to the largest size the checks above
  // allow and never lowered, so threads pruning different sizes at the same
  // time cannot undo each other's setting.
  st = ensure_smem_attr(ctx, kSmemPrune, prune_select_kernel, kPruneSelectSmemMax,
                        "prune smem attribute");
  if (st != SAM3_OK) return st;
  {
    ProfScope prof(ctx, SAM3_PROF_PRUNE, 0.0, 4.0 * rows + 4.0 * batch * keep);
    prune_select_kernel<<<batch, 1024, smem, ctx->stream>>>(scores, seq, keep, order, idx);
    if ((st = check_launch(ctx, "prune_select_kernel")) != SAM3_OK) return st;
  }
  const int total = batch * keep;
  ProfScope prof(ctx, SAM3_PROF_PRUNE, 0.0,
                 4.0 * total * d + (rope_in ? 8.0 * total * rope_cols : 0.0) + 4.0 * total);
  prune_gather_kernel<<<blocks_for(total, 8), 256, 0, ctx->stream>>>(
      reinterpret_cast<const __half*>(x), seq, d, keep, idx, rope_in, rope_rows > 0 ? rope_rows : 1,
      rope_cols, reinterpret_cast<__half*>(feats), rope_out, total);
  return check_launch(ctx, "prune_gather_kernel");
}

sam3_status_t patch_embed(sam3_ctx_t* ctx, const void* image, bool rgba, int batch, int h,
                          int w, const uint16_t* pw, const uint16_t* pb, int patch, int dim,
                          uint16_t* out, uint16_t* cols, uint16_t* wpad) {
  if (!image || !pw || !out || !cols || !wpad)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "patch_embed: null pointer");
  if (batch <= 0 || patch <= 0 || h % patch || w % patch || dim % 128)
    return set_error(ctx, SAM3_ERR_SHAPE, "patch_embed: bad shape");
  const int k = 3 * patch * patch;
  const int kp = (k + 63) / 64 * 64;
  const long long tokens = (long long)batch * (h / patch) * (w / patch);
  sam3_status_t st;
  if (tokens > 0x7FFFFFFFll) return set_error(ctx, SAM3_ERR_SHAPE, "patch_embed: too many tokens");
  {
    ProfScope prof(ctx, SAM3_PROF_PATCH, 0.0,
                   (rgba ? 16.0 / 3.0 : 2.0) * tokens * k + 2.0 * tokens * kp);
    if (rgba)
      im2col_kernel<true><<<(int)tokens, 128, 0, ctx->stream>>>(image, h, w, patch, kp,
                                                                 reinterpret_cast<__half*>(cols));
    else
      im2col_kernel<false><<<(int)tokens, 128, 0, ctx->stream>>>(image, h, w, patch, kp,
                                                                  reinterpret_cast<__half*>(cols));
    st = check_launch(ctx, "im2col_kernel");
    if (st != SAM3_OK) return st;
  }
  {
    ProfScope prof(ctx, SAM3_PROF_PATCH, 0.0, 2.0 * dim * k + 2.0 * dim * kp);
  pad_weight_kernel<<<blocks_for((long long)dim * kp, 256), 256, 0, ctx->stream>>>(
      reinterpret_cast<const __half*>(pw), dim, k, kp, reinterpret_cast<__half*>(wpad));
  if ((st = check_launch(ctx, "pad_weight_kernel")) != SAM3_OK) return st;
  }
  return gemm_dense(ctx, cols, (int)tokens, kp, wpad, pb, dim, out);
}

}  // namespace sam3

using namespace sam3;

extern "C" {

sam3_status_t sam3_layernorm(sam3_ctx_t* ctx, const uint16_t* x, int32_t m, int32_t d,
                             const uint16_t* gamma, const uint16_t* beta, float eps, uint16_t* y) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  return layernorm(ctx, x, m, d, gamma, beta, eps, y);
}

sam3_status_t sam3_rope_table(sam3_ctx_t* ctx, int32_t gh, int32_t gw, int32_t hd, float theta,
                              float* table) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  return rope_table(ctx, gh, gw, hd, theta, table);
}

sam3_status_t sam3_rope_apply(sam3_ctx_t* ctx, uint16_t* qkv, int32_t m, int32_t heads,
                              int32_t hd, const float* table, int32_t rope_rows) {
  SAM3_CHECK_CTX(ctx);
  if (!qkv || !table) return set_error(ctx, SAM3_ERR_INVALID_ARG, "rope_apply: null pointer");
  if (m <= 0 || heads <= 0 || hd <= 0 || hd % 2 || rope_rows <= 0)
    return set_error(ctx, SAM3_ERR_SHAPE, "rope_apply: bad shape");
  if (reinterpret_cast<uintptr_t>(qkv) & 3u)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "rope_apply: qkv must be 4-byte aligned");
  cudaSetDevice(ctx->device);
  const int dim = heads * hd;
  ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 8.0 * m * dim + 8.0 * m * hd / 2);
  rope_apply_kernel<<<blocks_for((long long)m * dim, 256), 256, 0, ctx->stream>>>(
      reinterpret_cast<__half2*>(qkv), m, dim, hd, reinterpret_cast<const float2*>(table),
      rope_rows);
  return check_launch(ctx, "rope_apply_kernel");
}

sam3_status_t sam3_token_scores(sam3_ctx_t* ctx, const uint16_t* x, int32_t rows, int32_t d,
                                int32_t norm, float* scores) {
  SAM3_CHECK_CTX(ctx);
  if (!x || !scores) return set_error(ctx, SAM3_ERR_INVALID_ARG, "token_scores: null pointer");
  if (rows <= 0 || d <= 0 || d % 8) return set_error(ctx, SAM3_ERR_SHAPE, "token_scores: bad shape");
  if (norm != SAM3_SCORE_L2 && norm != SAM3_SCORE_L1)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "token_scores: bad norm");
  if (!aligned16(x)) return set_error(ctx, SAM3_ERR_INVALID_ARG, "token_scores: x alignment");
  cudaSetDevice(ctx->device);
  ProfScope prof(ctx, SAM3_PROF_PRUNE, 0.0, 2.0 * rows * d + 4.0 * rows);
  token_score_kernel<<<blocks_for(rows, 8), 256, 0, ctx->stream>>>(
      reinterpret_cast<const __half*>(x), rows, d, norm, scores);
  return check_launch(ctx, "token_score_kernel");
}

sam3_status_t sam3_prune(sam3_ctx_t* ctx, const uint16_t* x, int32_t batch, int32_t seq, int32_t d,
                         int32_t keep, int32_t norm, int32_t order, const float* rope_in,
                         int32_t rope_rows, int32_t rope_cols, uint16_t* feats, float* rope_out,
                         int32_t* idx) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  if ((long long)batch * seq > (long long)ctx->block_rows) {
    // scores scratch lives in the workspace; grow it outside any hot loop
    return set_error(ctx, SAM3_ERR_SHAPE, "prune: batch*seq=%lld exceeds context capacity %zu",
                     (long long)batch * seq, ctx->block_rows);
  }
  return prune(ctx, x, batch, seq, d, keep, norm, order, rope_in, rope_rows, rope_cols, feats,
               rope_out, idx, ctx->scores);
}

sam3_status_t sam3_patch_embed(sam3_ctx_t* ctx, const uint16_t* image, int32_t batch, int32_t h,
                               int32_t w, const uint16_t* pw, const uint16_t* pb, int32_t patch,
                               int32_t dim, uint16_t* out) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  const int k = 3 * patch * patch, kp = (k + 63) / 64 * 64;
  const size_t tokens = (size_t)batch * (h / (patch > 0 ? patch : 1)) * (w / (patch > 0 ? patch : 1));
  const sam3_encoder_config_t& c = ctx->cfg;
  const size_t cap_cols = ctx->block_rows * (size_t)((3 * c.patch * c.patch + 63) / 64 * 64);
  if (patch <= 0 || tokens * kp > cap_cols || (size_t)dim * kp > (size_t)c.embed_dim *
                                                                     ((3 * c.patch * c.patch + 63) / 64 * 64))
    return set_error(ctx, SAM3_ERR_SHAPE, "patch_embed: shape exceeds context workspace");
  return patch_embed(ctx, image, false, batch, h, w, pw, pb, patch, dim, out, ctx->cols,
                     ctx->patch_wp);
}

sam3_status_t sam3_patch_embed_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch, int32_t h,
                                    int32_t w, const uint16_t* pw, const uint16_t* pb,
                                    int32_t patch, int32_t dim, uint16_t* out) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  const int k = 3 * patch * patch, kp = (k + 63) / 64 * 64;
  const size_t tokens = (size_t)batch * (h / (patch > 0 ? patch : 1)) * (w / (patch > 0 ? patch : 1));
  const sam3_encoder_config_t& c = ctx->cfg;
  const size_t cap_cols = ctx->block_rows * (size_t)((3 * c.patch * c.patch + 63) / 64 * 64);
  if (patch <= 0 || tokens * kp > cap_cols || (size_t)dim * kp > (size_t)c.embed_dim *
                                                                     ((3 * c.patch * c.patch + 63) / 64 * 64))
    return set_error(ctx, SAM3_ERR_SHAPE, "patch_embed: shape exceeds context workspace");
  if (!rgba || !aligned16(rgba))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "patch_embed: rgba must be a 16-byte aligned pointer");
  return patch_embed(ctx, rgba, true, batch, h, w, pw, pb, patch, dim, out, ctx->cols,
                     ctx->patch_wp);
}

sam3_status_t sam3_preprocess_rgba(sam3_ctx_t* ctx, const float* rgba, int32_t batch,
                                   int32_t height, int32_t width, uint16_t* rgb) {
  SAM3_CHECK_CTX(ctx);
  cudaSetDevice(ctx->device);
  if (!rgba || !rgb) return set_error(ctx, SAM3_ERR_INVALID_ARG, "preprocess: null pointer");
  if (!aligned16(rgba)) return set_error(ctx, SAM3_ERR_INVALID_ARG, "preprocess: rgba must be 16-byte aligned");
  if (batch <= 0 || height <= 0 || width <= 0)
    return set_error(ctx, SAM3_ERR_SHAPE, "preprocess: empty shape");
  const long long pixels = (long long)batch * height * width;
  ProfScope prof(ctx, SAM3_PROF_PATCH, 0.0, 22.0 * pixels);
  const int grid = (int)std::min<long long>((pixels + 255) / 256, (long long)ctx->num_sms * 16);
  preprocess_rgba_kernel<<<grid, 256, 0, ctx->stream>>>(reinterpret_cast<const float4*>(rgba),
                                                        pixels, reinterpret_cast<__half*>(rgb));
  return check_launch(ctx, "preprocess_rgba_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free pruning
// The score scratch of sam3_prune_noalloc lives in this fixed device array
// instead of a context workspace. Every GPU that loads the library holds it
// (SAM3_PRUNE_NOALLOC_MAX_ROWS floats) until the process exits.
namespace {
static __device__ __align__(256) float g_noalloc_scores[SAM3_PRUNE_NOALLOC_MAX_ROWS];
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
// Per device: the array's device address and whether prune_select_kernel's
// shared-memory limit has been raised there. Looked up once per device; a
// cudaDeviceReset of that device invalidates them (see the header).
float* g_noalloc_addr[kMaxDevices] = {};
bool g_noalloc_smem[kMaxDevices] = {};

// Switches to `dev` for the lifetime of the scope when it is not current.
struct DeviceScope {
  int prev = -1;
  bool ok = true;
  explicit DeviceScope(int dev) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) { ok = false; return; }
    if (cur != dev) {
      if (cudaSetDevice(dev) != cudaSuccess) { ok = false; return; }
      prev = cur;
    }
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" sam3_status_t sam3_prune_noalloc(void* cuda_stream, const uint16_t* x, int32_t batch,
                                            int32_t seq, int32_t d, int32_t keep, int32_t norm,
                                            int32_t order, const float* rope_in,
                                            int32_t rope_rows, int32_t rope_cols,
                                            uint16_t* feats, float* rope_out, int32_t* idx) {
  if (!x || !feats || !idx) return SAM3_ERR_INVALID_ARG;
  if (batch <= 0 || seq <= 0 || d <= 0 || d % 8 || keep <= 0 || keep > seq || seq > 16384)
    return SAM3_ERR_SHAPE;
  if ((long long)batch * seq > SAM3_PRUNE_NOALLOC_MAX_ROWS) return SAM3_ERR_SHAPE;
  if (norm != SAM3_SCORE_L2 && norm != SAM3_SCORE_L1) return SAM3_ERR_INVALID_ARG;
  if (order != SAM3_ORDER_INDEX && order != SAM3_ORDER_SCORE) return SAM3_ERR_INVALID_ARG;
  if (order == SAM3_ORDER_SCORE && keep > 8192) return SAM3_ERR_SHAPE;
  if ((rope_in == nullptr) != (rope_out == nullptr) ||
      (rope_in && (rope_rows <= 0 || rope_cols <= 0)))
    return SAM3_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(feats)) return SAM3_ERR_INVALID_ARG;

  // An error already pending on this thread belongs to earlier work: it is
  // left in place, and only errors of this call's own runtime calls are
  // cleared (each of those returns its error directly).
  const bool clean_before = cudaPeekAtLastError() == cudaSuccess;
  auto fail = [clean_before]() {
    if (clean_before) cudaGetLastError();
    return SAM3_ERR_CUDA;
  };

  // The work runs on the stream's device (the current device for the legacy
  // default stream), which is made current for the call.
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  int dev = -1;
  if (stream == nullptr ? cudaGetDevice(&dev) != cudaSuccess
                        : cudaStreamGetDevice(stream, &dev) != cudaSuccess)
    return fail();
  if (dev < 0 || dev >= kMaxDevices) return SAM3_ERR_UNSUPPORTED;
  DeviceScope on_dev(dev);
  if (!on_dev.ok) return fail();

  // Set-up, once per device with that device current: the host-side name of
  // a __device__ array is only a stand-in, so ask the runtime for its device
  // address and hand that to the kernels. prune_select_kernel's dynamic
  // shared-memory limit is raised there once, to the largest size accepted
  // above, and never lowered.
  float* scores = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scores) != cudaSuccess || !p) return fail();
      g_noalloc_addr[dev] = static_cast<float*>(p);
    }
    if (!g_noalloc_smem[dev]) {
      if (cudaFuncSetAttribute(prune_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kPruneSelectSmemMax) != cudaSuccess)
        return fail();
      g_noalloc_smem[dev] = true;
    }
    scores = g_noalloc_addr[dev];
  }

  const long long rows = (long long)batch * seq;
  // Every score is rewritten before it is read, so nothing needs clearing.
  if (launch_plain(token_score_kernel, dim3(blocks_for(rows, 8)), dim3(256), 0, stream,
                   reinterpret_cast<const __half*>(x), (int)rows, (int)d, (int)norm,
                   scores) != cudaSuccess)
    return fail();
  size_t smem = ((size_t)seq * 4 + 15) & ~(size_t)15;
  if (order == SAM3_ORDER_SCORE) {
    int p2 = 1;
    while (p2 < keep) p2 <<= 1;
    smem += (size_t)p2 * 8;
  }
  if (launch_plain(prune_select_kernel, dim3(batch), dim3(1024), smem, stream,
                   static_cast<const float*>(scores), (int)seq, (int)keep, (int)order,
                   idx) != cudaSuccess)
    return fail();
  const int total = batch * keep;
  if (launch_plain(prune_gather_kernel, dim3(blocks_for(total, 8)), dim3(256), 0, stream,
                   reinterpret_cast<const __half*>(x), (int)seq, (int)d, (int)keep,
                   static_cast<const int32_t*>(idx), rope_in, rope_rows > 0 ? (int)rope_rows : 1,
                   (int)rope_cols, reinterpret_cast<__half*>(feats), rope_out,
                   total) != cudaSuccess)
    return fail();
  return SAM3_OK;
}
