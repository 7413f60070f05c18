// attention.cu - global softmax attention over packed QKV rows.
//
// o[b*S + i, h*64 + :] = softmax_j(q_i . k_j * scale) v_j, per image b and
// head h, reading q | k | v straight from the QKV GEMM output
// [B*S, 3*H*64] (no transpose pass) and writing the [B*S, H*64] layout the
// out-projection GEMM consumes.
//
// Reference: scaledDotProductAttention in MPSAttentionLayer
// (MPSAttention.swift:165-176, scale 1/sqrt(64), no mask) and the explicit
// QK^T -> softmax -> PV form of AttentionKernels.swift:48-68.
//
// Flash-style single pass: a CTA owns 128 query rows of one (image, head);
// 8 warps x 16 rows; 64-key K/V tiles stream through a cp.async double
// buffer in 128B-XOR-swizzled shared memory; fp16 m16n8k16 tensor-core MMAs
// with fp32 accumulation; online softmax in fp32 (exp2 with the scale folded
// into log2 e); P is rounded to fp16 for the PV product.
#include <stdlib.h>

#include "common.cuh"
#include "internal.h"

namespace sam3 {
sam3_status_t attention_tc(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                           float scale, uint16_t* o);
namespace {

constexpr int HD = 64;
constexpr int BQ = 128, BKV = 64, THREADS = 256;

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(THREADS) flash_attn_kernel(const __half* __restrict__ qkv,
                                                             int seq, int heads, float scale_log2,
                                                             __half* __restrict__ out) {
  __shared__ __align__(128) uint8_t sq[BQ * HD * 2];
  __shared__ __align__(128) uint8_t sk[2][BKV * HD * 2];
  __shared__ __align__(128) uint8_t sv[2][BKV * HD * 2];

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int dim = heads * HD;
  const size_t row_stride = 3 * (size_t)dim;
  const __half* base = qkv + (size_t)b * seq * row_stride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sq_a = smem_u32(sq);
  const uint32_t sk_a[2] = {smem_u32(sk[0]), smem_u32(sk[1])};
  const uint32_t sv_a[2] = {smem_u32(sv[0]), smem_u32(sv[1])};

  // Q tile: 128 rows x 8 chunks of 16 B.
#pragma unroll
  for (int it = 0; it < (BQ * 8) / THREADS; ++it) {
    const int c = tid + it * THREADS;
    const int r = c >> 3, ch = c & 7;
    const int q = qt * BQ + r;
    const bool valid = q < seq;
    const __half* src = base + (size_t)(valid ? q : 0) * row_stride + h * HD + ch * 8;
    cp_async16(sq_a + swz(r, ch), src, valid);
  }
  auto load_kv = [&](int tile, int buf) {
#pragma unroll
    for (int it = 0; it < (BKV * 8) / THREADS; ++it) {
      const int c = tid + it * THREADS;
      const int r = c >> 3, ch = c & 7;
      const int kv = tile * BKV + r;
      const bool valid = kv < seq;
      const __half* src = base + (size_t)(valid ? kv : 0) * row_stride + dim + h * HD + ch * 8;
      cp_async16(sk_a[buf] + swz(r, ch), src, valid);
      cp_async16(sv_a[buf] + swz(r, ch), src + dim, valid);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const int ntiles = (seq + BKV - 1) / BKV;
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) load_kv(j + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(sq_a + swz(r, ch), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
      }
    }
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int mi = lane >> 3;
        const int r = np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int ch = kk * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sk_a[buf] + swz(r, ch), b0, b1, b2, b3);
        mma16816(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
        mma16816(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
      }
    }
    // mask keys past the end, scale into log2 domain, online softmax
    const int key0 = j * BKV;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + nt * 8 + 2 * t4 + (e & 1);
        const float v = key < seq ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], mnew[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(m_r[r], mx[r]);
      alpha[r] = exp2f(m_r[r] - mnew[r]);  // m_r = -inf on the first tile -> 0
      m_r[r] = mnew[r];
    }
    uint32_t pa[8][2];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mnew[0]), p1 = exp2f(s[nt][1] - mnew[0]);
      const float p2 = exp2f(s[nt][2] - mnew[1]), p3 = exp2f(s[nt][3] - mnew[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      pa[nt][0] = pack_half2(p0, p1);
      pa[nt][1] = pack_half2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_r[r] = l_r[r] * alpha[r] + rs[r];
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      o[dt][0] *= alpha[0];
      o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1];
      o[dt][3] *= alpha[1];
    }
    // O += P V: k-steps of 16 keys, d-tiles of 8.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int mi = lane >> 3;
        const int r = kk * 16 + (lane & 7) + (mi & 1) * 8;
        const int ch = dp * 2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sv_a[buf] + swz(r, ch), b0, b1, b2, b3);
        mma16816(o[2 * dp], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0], pa[2 * kk + 1][1],
                 b0, b1);
        mma16816(o[2 * dp + 1], pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0],
                 pa[2 * kk + 1][1], b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // finalize: row sums across the quad, normalise, store fp16
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  const float inv0 = 1.f / l_r[0], inv1 = 1.f / l_r[1];
  const int q0 = qt * BQ + warp * 16 + g;
  __half* ob = out + (size_t)b * seq * dim + h * HD;
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    const int col = dt * 8 + 2 * t4;
    if (q0 < seq)
      *reinterpret_cast<uint32_t*>(ob + (size_t)q0 * dim + col) =
          pack_half2(o[dt][0] * inv0, o[dt][1] * inv0);
    if (q0 + 8 < seq)
      *reinterpret_cast<uint32_t*>(ob + (size_t)(q0 + 8) * dim + col) =
          pack_half2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

}  // namespace

sam3_status_t attention(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                        int head_dim, float scale, uint16_t* o) {
  if (!qkv || !o) return set_error(ctx, SAM3_ERR_INVALID_ARG, "attention: null pointer");
  if (head_dim != HD)
    return set_error(ctx, SAM3_ERR_SHAPE, "attention: head_dim must be 64 (got %d)", head_dim);
  if (batch <= 0 || seq <= 0 || heads <= 0 || heads > 65535 || batch > 65535)
    return set_error(ctx, SAM3_ERR_SHAPE, "attention: bad shape");
  if (!aligned16(qkv) || !aligned16(o))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "attention: pointers must be 16-byte aligned");
  static const bool legacy = [] {
    const char* v = getenv("SAM3_ATTENTION_MMA_SYNC");
    return v && v[0] == '1';
  }();
  if (!legacy) {
    ProfScope prof(ctx, SAM3_PROF_ATTENTION, 4.0 * batch * heads * (double)seq * seq * HD,
                   8.0 * batch * seq * heads * HD);
    return attention_tc(ctx, qkv, batch, seq, heads, scale, o);
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((seq + BQ - 1) / BQ, heads, batch);
  ProfScope prof(ctx, SAM3_PROF_ATTENTION, 4.0 * batch * heads * (double)seq * seq * HD,
                 8.0 * batch * seq * heads * HD);
  flash_attn_kernel<<<grid, THREADS, 0, ctx->stream>>>(reinterpret_cast<const __half*>(qkv), seq,
                                                       heads, scale_log2,
                                                       reinterpret_cast<__half*>(o));
  return check_launch(ctx, "flash_attn_kernel");
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
