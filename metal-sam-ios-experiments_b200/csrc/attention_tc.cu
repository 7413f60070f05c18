// attention_tc.cu - global softmax attention on the sm_100a tensor cores
// (tcgen05 MMAs with tensor-memory accumulators, TMA-fed K/V stages).
//
// o[b*S + i, h*64 + :] = softmax_j(q_i . k_j * scale) v_j for every image b
// and head h, read straight from the packed QKV GEMM output [B*S, 3*H*64].
// Reference: scaledDotProductAttention (MPSAttention.swift:165-176, scale
// 1/sqrt(64), no mask) and AttentionKernels.swift:48-68 (explicit form).
//
// One CTA = 128 query rows of one (image, head); two CTAs per SM. Keys come
// in tiles of 64 and S is double-buffered in tensor memory, so Q K^T of tile
// j+2 is queued while the softmax works on tile j+1. Warp roles:
//   warp 0   TMA producer: Q tile once, then K/V tiles of 64 keys through a
//            3-stage ring (128B-swizzled, straight from the packed rows).
//   warp 1   TMEM allocator + single-thread MMA issuer:
//              S = Q K^T        (M=128, N=64, K=64, both operands K-major)
//              O += P [V | 1]   (M=128, N=80, K=64, P read from tensor
//                                memory, V as an MN-major operand followed by
//                                a constant block of ones)
//   warps 2-5  one thread per query row (its TMEM lane): the row's scores
//            read once, row max over the valid keys (three-input max),
//            p = 2^(s*scale*log2e - m) rounded to fp16 and written back over S
//            in tensor memory. The ones columns make the tensor core keep the
//            row sums of the fp16 P (O column 64), so the softmax threads add
//            nothing up and the normaliser has exactly the rounding of the P
//            that multiplied V. O stays in tensor memory and is rescaled in
//            place only when the running max grows by more than 8 (log2).
// Tensor memory (256 columns): S/P buffers at [0,64) and [64,128), O and the
// row sums at [128,208).
#include "common.cuh"
#include "internal.h"

namespace sam3 {
namespace {

constexpr int HD = 64, BQ = 128, BKV = 64, STAGES = 3;
constexpr int THREADS = 192;
constexpr int Q_BYTES = BQ * HD * 2;    // 16 KB
constexpr int KV_BYTES = BKV * HD * 2;  // 8 KB per K or V tile
constexpr int OFF_Q = 0;
// A K/V stage is 24 KB: the K tile, the V tile (one 3-D TMA request brings
// both), then an 8 KB block of fp16 ones that the PV MMA reads as 16 extra B
// columns (the row sums of P land in O column 64).
constexpr int KV_STAGE = 3 * KV_BYTES;
constexpr int OFF_KV = OFF_Q + Q_BYTES;
constexpr int OFF_BAR = OFF_KV + STAGES * KV_STAGE;
constexpr int NUM_BARS = 1 + 2 * STAGES + 2 + 2 + 1 + 1 + 1;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t COL_S0 = 0, COL_O = 128;  // S/P buffers at 0 and 64, O at 128
constexpr uint32_t IDESC_S = umma_idesc_f16(128, BKV, 0);  // K-major B (keys x d)
constexpr int OW = HD + 16;                                // O columns: d, then sum(P)
constexpr uint32_t IDESC_O = umma_idesc_f16(128, OW, 1);   // MN-major B (keys x (d | 1))

struct AttnArgs {
  __half* out;
  int* err;
  int seq, heads, dim;
  // grid.z item z attends over rows [row0, row0 + seq) of the packed QKV:
  // row0 = (z / groups) * img_rows + first_row + (z % groups) * seq (one
  // group per image for plain attention; windows of an image otherwise)
  int groups, img_rows, first_row;
  float scale_log2;
  int kv3d;  // 1: tmap_kv is the 3-D K|V map (one request per stage), 0: use 2-D boxes
  int o32;   // out is 32-byte aligned (256-bit stores)
};

// B descriptor of the PV MMA: V (MN-major, 128B swizzle) with the ones block
// one 64-column group further (leading byte offset = one tile, 8 KB).
__device__ __forceinline__ uint64_t desc_v_ones(uint32_t saddr) {
  return (umma_desc_sw128_mn(saddr) & ~(0x3FFFull << 16)) |
         (static_cast<uint64_t>(KV_BYTES >> 4) << 16);
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__global__ void __launch_bounds__(THREADS, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_qkv,
                   const __grid_constant__ CUtensorMap tmap_kv, const AttnArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int seq = args.seq, dim = args.dim;
  const int row0 = (b / args.groups) * args.img_rows + args.first_row + (b % args.groups) * seq;
  const int q0 = qt * BQ;
  const int ntiles = (seq + BKV - 1) / BKV;

  const uint32_t bar_q = sbase + OFF_BAR;
  const uint32_t bar_kv_full = bar_q + 8;
  const uint32_t bar_kv_empty = bar_kv_full + 8 * STAGES;
  const uint32_t bar_s_full = bar_kv_empty + 8 * STAGES;  // [2], per S buffer
  // [2], per S buffer: tile j completes phase j/2 of p_full[j%2]. (A single
  // barrier could alias: the softmax may finish tiles j and j+1 before the
  // MMA thread waits for tile j.)
  const uint32_t bar_p_full = bar_s_full + 16;
  const uint32_t bar_o_full = bar_p_full + 16;
  const uint32_t bar_drain = bar_o_full + 8;
  // Completes once, after the last PV: the read-out of O cannot use a parity
  // wait on o_full, whose phase may still be two behind at that point.
  const uint32_t bar_o_done = bar_drain + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_kv_full + 8 * s, 1);
      mbar_init(bar_kv_empty + 8 * s, 1);
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_full + 8, 1);
    mbar_init(bar_p_full, 128);
    mbar_init(bar_p_full + 8, 128);
    mbar_init(bar_o_full, 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_o_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_qkv);
    prefetch_tmap(&tmap_kv);
  }
  for (int i = threadIdx.x; i < STAGES * KV_BYTES / 16; i += THREADS) {  // fp16 1.0 blocks
    const int st = i / (KV_BYTES / 16), w = i % (KV_BYTES / 16);
    reinterpret_cast<uint4*>(smem + OFF_KV + st * KV_STAGE + 2 * KV_BYTES)[w] =
        make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      griddep_wait();  // Q/K/V are the previous kernel's output
      uint32_t issued = 0, issued_par = 0;
      mbar_arrive_expect_tx(bar_q, Q_BYTES);
      tma_load_2d(sbase + OFF_Q, &tmap_qkv, bar_q, h * HD, row0 + q0);
      tma_load_2d(sbase + OFF_Q + KV_BYTES, &tmap_qkv, bar_q, h * HD, row0 + q0 + BKV);
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (uint32_t)(j / STAGES) & 1u;
        if (!mbar_wait(bar_kv_empty + 8 * s, ph ^ 1, abort_flag, args.err, kDevErrTimeoutAttn))
          break;
        mbar_arrive_expect_tx(bar_kv_full + 8 * s, 2 * KV_BYTES);
        const int r = row0 + j * BKV;
        const uint32_t dst = sbase + OFF_KV + s * KV_STAGE;
        if (args.kv3d) {
          tma_load_3d(dst, &tmap_kv, bar_kv_full + 8 * s, h * HD, r, 0);
        } else {
          tma_load_2d(dst, &tmap_qkv, bar_kv_full + 8 * s, dim + h * HD, r);
          tma_load_2d(dst + KV_BYTES, &tmap_qkv, bar_kv_full + 8 * s, 2 * dim + h * HD, r);
        }
        issued |= 1u << s;
        issued_par = (issued_par & ~(1u << s)) | (ph << s);
      }
      if (*abort_flag) {
        mbar_wait_drain(bar_q, 0);
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait_drain(bar_kv_full + 8 * s, (issued_par >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    // Order: S0 = Q K0^T, S1 = Q K1^T, then per tile j: O += P_j V_j and,
    // once that PV has read P_j, S_(j%2) = Q K_(j+2)^T.
    if (lane == 0) {
      bool issued_any = false, ok = true;
      const uint64_t dq = umma_desc_sw128(sbase + OFF_Q);
      auto issue_qk = [&](int j) -> bool {
        const int s = j % STAGES;
        if (!mbar_wait(bar_kv_full + 8 * s, (uint32_t)(j / STAGES) & 1u, abort_flag, args.err,
                       kDevErrTimeoutAttn))
          return false;
        tc_fence_after();
        const uint64_t dk = umma_desc_sw128(sbase + OFF_KV + s * KV_STAGE);
        const uint32_t d = tmem + COL_S0 + (uint32_t)((j & 1) * BKV);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16_ss(d, desc_advance(dq, kk * 32), desc_advance(dk, kk * 32), IDESC_S, kk != 0);
        umma_commit(bar_s_full + 8 * (j & 1));
        issued_any = true;
        return true;
      };
      ok = mbar_wait(bar_q, 0, abort_flag, args.err, kDevErrTimeoutAttn);
      if (ok) ok = issue_qk(0);
      if (ok && ntiles > 1) ok = issue_qk(1);
      for (int j = 0; j < ntiles && ok; ++j) {
        const int s = j % STAGES;
        if (!mbar_wait(bar_p_full + 8 * (j & 1), (uint32_t)(j >> 1) & 1u, abort_flag, args.err,
                       kDevErrTimeoutAttn))
          break;
        tc_fence_after();
        const uint64_t dv = desc_v_ones(sbase + OFF_KV + s * KV_STAGE + KV_BYTES);
        const uint32_t p_col = tmem + COL_S0 + (uint32_t)((j & 1) * BKV);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_f16_ts(tmem + COL_O, p_col + kk * 8, desc_advance(dv, kk * 2048), IDESC_O,
                      (j | kk) != 0);
        umma_commit(bar_o_full);
        umma_commit(bar_kv_empty + 8 * s);
        if (j == ntiles - 1) umma_commit(bar_o_done);
        if (j + 2 < ntiles) {
          // S_(j%2) holds P_j until this PV has read it
          if (!mbar_wait(bar_o_full, (uint32_t)j & 1u, abort_flag, args.err, kDevErrTimeoutAttn))
            break;
          ok = issue_qk(j + 2);
        }
      }
      if (*abort_flag && issued_any) {
        umma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------- softmax rows
    // One thread per query row (its TMEM lane): the tile's 64 scores are read
    // once; p = 2^(s*scale*log2e - m) rounded to fp16 overwrites S as P; O
    // accumulates in tensor memory and is rescaled in place only when the
    // running max grows by more than kRescaleLog2 (so p <= 2^8, exact in fp16).
    constexpr float kRescaleLog2 = 8.0f;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float c = args.scale_log2;
    float m_run = -INFINITY;
    bool ok = true;
    griddep_wait();  // before this grid's output rows are written
    for (int j = 0; j < ntiles && ok; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full + 8 * (j & 1), (uint32_t)(j >> 1) & 1u,
                                             abort_flag, args.err, kDevErrTimeoutAttn));
      if (!ok) break;
      tc_fence_after();
      const uint32_t s_col = lane_base + COL_S0 + (uint32_t)((j & 1) * BKV);
      uint32_t v[BKV];
      tmem_ld_32x32b_x32(s_col, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_32x32b_x32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_wait_ld();
      const int valid = min(BKV, seq - j * BKV);  // only the last tile can be ragged
      if (valid < BKV) {
#pragma unroll
        for (int e = 0; e < BKV; ++e)
          if (e >= valid) v[e] = __float_as_uint(-INFINITY);
      }
      float mx0 = __uint_as_float(v[0]), mx1 = __uint_as_float(v[32]);
#pragma unroll
      for (int e = 1; e < 31; e += 2) {
        mx0 = max3f(mx0, __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
        mx1 = max3f(mx1, __uint_as_float(v[32 + e]), __uint_as_float(v[32 + e + 1]));
      }
      const float m_tile = max3f(fmaxf(mx0, __uint_as_float(v[31])), mx1, __uint_as_float(v[63])) * c;
      const bool grow = m_tile > m_run + kRescaleLog2;
      const float m_use = grow ? m_tile : m_run;
      const float alpha = grow ? ex2_approx(m_run - m_use) : 1.0f;  // 0 on the first tile
#pragma unroll
      for (int cc = 0; cc < BKV / 32; ++cc) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(v[cc * 32 + 2 * e]), c, -m_use));
          const float p1 = ex2_approx(fmaf(__uint_as_float(v[cc * 32 + 2 * e + 1]), c, -m_use));
          pk[e] = pack_half2(p0, p1);
        }
        tmem_st_32x32b_x16(s_col + cc * 16, pk);
      }
      m_run = m_use;
      // The rescale uses warp-collective tcgen05.ld/st, so the whole warp takes
      // the branch when any of its rows grew (alpha is 1 for the others).
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // wait for the previous tiles' sum, then rescale the rows in place
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o_full, (uint32_t)(j - 1) & 1u, abort_flag,
                                               args.err, kDevErrTimeoutAttn));
        if (!ok) break;
        tc_fence_after();
        uint32_t o[OW];
        tmem_ld_32x32b_x32(lane_base + COL_O, *reinterpret_cast<uint32_t(*)[32]>(o));
        tmem_ld_32x32b_x32(lane_base + COL_O + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
        tmem_ld_32x32b_x16(lane_base + COL_O + 64, *reinterpret_cast<uint32_t(*)[16]>(o + 64));
        tmem_wait_ld();
#pragma unroll
        for (int d = 0; d < OW; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * alpha);
#pragma unroll
        for (int q = 0; q < OW / 16; ++q)
          tmem_st_32x32b_x16(lane_base + COL_O + q * 16, *reinterpret_cast<uint32_t(*)[16]>(o + 16 * q));
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p_full + 8 * (j & 1));
    }
    if (ok)
      ok = __all_sync(0xffffffffu, mbar_wait(bar_o_done, 0u, abort_flag,
                                             args.err, kDevErrTimeoutAttn));
    if (ok) {
      tc_fence_after();
      uint32_t o[OW];
      tmem_ld_32x32b_x32(lane_base + COL_O, *reinterpret_cast<uint32_t(*)[32]>(o));
      tmem_ld_32x32b_x32(lane_base + COL_O + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
      tmem_ld_32x32b_x16(lane_base + COL_O + 64, *reinterpret_cast<uint32_t(*)[16]>(o + 64));
      tmem_wait_ld();
      const int q = q0 + r;
      if (q < seq) {
        const float inv = 1.f / __uint_as_float(o[HD]);  // sum of P, from the ones columns
        __half* drow = args.out + (size_t)(row0 + q) * dim + h * HD;
        if (args.o32) {  // 32-byte stores: whole sectors, half the instructions
#pragma unroll
          for (int c16 = 0; c16 < HD / 16; ++c16) {
            uint32_t w[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              w[e] = pack_half2(__uint_as_float(o[16 * c16 + 2 * e]) * inv,
                                __uint_as_float(o[16 * c16 + 2 * e + 1]) * inv);
            st_global_v8(drow + 16 * c16, w);
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(drow);
#pragma unroll
          for (int c8 = 0; c8 < HD / 8; ++c8) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(o[8 * c8 + 0]) * inv, __uint_as_float(o[8 * c8 + 1]) * inv);
            w.y = pack_half2(__uint_as_float(o[8 * c8 + 2]) * inv, __uint_as_float(o[8 * c8 + 3]) * inv);
            w.z = pack_half2(__uint_as_float(o[8 * c8 + 4]) * inv, __uint_as_float(o[8 * c8 + 5]) * inv);
            w.w = pack_half2(__uint_as_float(o[8 * c8 + 6]) * inv, __uint_as_float(o[8 * c8 + 7]) * inv);
            dst[c8] = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

sam3_status_t attention_tc(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                           float scale, uint16_t* o, int groups, int img_rows, int first_row) {
  const int dim = heads * HD;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)(3 * dim), (cuuint64_t)batch * img_rows};
  cuuint64_t strides[1] = {(cuuint64_t)(3 * dim) * 2};
  cuuint32_t box[2] = {HD, BKV};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_tiled()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(qkv),
                              dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, SAM3_ERR_CUDA, "attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
  // K and V of all heads as a 3-D tensor (dim columns, B*S rows, {k, v}): the
  // box {64, BKV, 2} is one head's K tile followed by its V tile.
  CUtensorMap map_kv;
  cuuint64_t dims3[3] = {(cuuint64_t)dim, (cuuint64_t)batch * img_rows, 2};
  cuuint64_t strides3[2] = {(cuuint64_t)(3 * dim) * 2, (cuuint64_t)dim * 2};
  cuuint32_t box3[3] = {HD, BKV, 2};
  cuuint32_t es3[3] = {1, 1, 1};
  const bool kv3d =
      encode_tiled()(&map_kv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t*>(qkv + dim),
                     dims3, strides3, box3, es3, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  const sam3_status_t st =
      ensure_smem_attr(ctx, kSmemAttn, attn_tc_kernel, SMEM_BYTES, "attention smem attribute");
  if (st != SAM3_OK) return st;
  AttnArgs a;
  a.out = reinterpret_cast<__half*>(o);
  a.err = ctx->dev_err;
  a.seq = seq;
  a.groups = groups;
  a.img_rows = img_rows;
  a.first_row = first_row;
  a.heads = heads;
  a.dim = dim;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.kv3d = kv3d ? 1 : 0;
  a.o32 = (reinterpret_cast<uintptr_t>(o) & 31u) == 0;
  dim3 grid((seq + BQ - 1) / BQ, heads, batch * groups);
  const cudaError_t e = launch_pdl(attn_tc_kernel, grid, dim3(THREADS), SMEM_BYTES, ctx->stream,
                                   map, kv3d ? map_kv : map, a);
  return check_launch_ret(ctx, e, "attn_tc_kernel");
}

}  // namespace sam3
