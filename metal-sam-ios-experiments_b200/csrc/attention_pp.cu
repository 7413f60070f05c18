// attention_pp.cu - global softmax attention on the sm_100a tensor cores with
// 128-key tiles and the scores double-buffered through registers.
//
// o[b*S + i, h*64 + :] = softmax_j(q_i . k_j * scale) v_j for every image b
// and head h, read straight from the packed QKV GEMM output [B*S, 3*H*64].
// Reference: scaledDotProductAttention (MPSAttention.swift:165-176, scale
// 1/sqrt(64), no mask) and AttentionKernels.swift:48-68 (explicit form).
//
// One CTA owns 128 query rows of one (image, head); two CTAs share an SM
// (97 KB of shared memory and 256 TMEM columns each), so the two CTAs'
// softmax phases drift apart and interleave on the MUFU. Keys come in tiles
// of 128 (K through a 3-deep ring, V through a 2-deep one). Warp roles
// (192 threads):
//   warp 0     TMA producer: Q once; then per key tile its K tile and its V
//              tile straight from the packed rows.
//   warp 1     TMEM allocator + single-thread MMA issuer:
//                S = Q K^T   (M=128, N=128, K=64; both K-major)
//                O += P V    (M=128, N=64, K=128; P from tensor memory,
//                             V MN-major)
//   warps 2-5  softmax: one thread per query row (its TMEM lane) loads the
//              row's 128 scores into registers and releases S at once, so
//              Q K^T of the next key tile runs while this tile's
//              exponentials are computed; p = 2^(s*scale*log2e - m) rounded to
//              fp16 into P (its own 64 columns), and the row sum of p in
//              registers. O is rescaled in place only when the running max
//              grows by more than 8 (log2), so p <= 2^8 stays exact enough in
//              fp16. The stores of P wait for PV(j-1), which completes while
//              the exponentials are computed.
// Issue order per key tile j: PV(j) as soon as P(j) is written, then QK(j+2)
// once the softmax has loaded S(j+1) into registers.
// Tensor memory (256 columns): S [0,128), P [128,192), O [192,256).
#include "common.cuh"
#include "internal.h"

namespace sam3 {
namespace {

constexpr int HD = 64, BQ = 128, BKV = 128;
// K tiles through a 3-deep ring (Q K^T runs a key tile ahead), V tiles
// through a 2-deep one.
constexpr int KST = 3, VST = 2;
constexpr int THREADS = 192;
constexpr int Q_BYTES = BQ * HD * 2;     // 16 KB
constexpr int KV_TILE = BKV * HD * 2;    // 16 KB per K or V tile
constexpr int OFF_Q = 0;
constexpr int OFF_K = Q_BYTES;
constexpr int OFF_V = OFF_K + KST * KV_TILE;
constexpr int OFF_BAR = OFF_V + VST * KV_TILE;
// q_full, k_full[KST], k_empty[KST], v_full[VST], v_empty[VST], s_full,
// s_free, p_full, o_full, o_done, drain
constexpr int NUM_BARS = 1 + 2 * KST + 2 * VST + 6;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
// two CTAs per SM (256 TMEM columns each), never three
static_assert(2 * (SMEM_BYTES + 1024) <= 228 * 1024 && 3 * SMEM_BYTES > 228 * 1024,
              "exactly two CTAs per SM");
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t COL_S = 0, COL_P = 128, COL_O = 192;
constexpr uint32_t IDESC_S = umma_idesc_f16(128, BKV, 0);  // K-major B (keys x d)
constexpr uint32_t IDESC_O = umma_idesc_f16(128, HD, 1);   // MN-major B (keys x d)

struct PPArgs {
  __half* out;
  int* err;
  int seq, heads, dim;
  int groups, img_rows, first_row;  // as in attention_tc.cu (one group per image here)
  float scale_log2;
  int o32;  // out is 32-byte aligned (256-bit stores)
};

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__global__ void __launch_bounds__(THREADS, 2)
    attn_pp_kernel(const __grid_constant__ CUtensorMap tmap_q, const PPArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int seq = args.seq, dim = args.dim;
  const int row0 = (b / args.groups) * args.img_rows + args.first_row + (b % args.groups) * seq;
  const int q0 = blockIdx.x * BQ;
  const int ntiles = (seq + BKV - 1) / BKV;

  const uint32_t bar_q = sbase + OFF_BAR;
  const uint32_t bar_k_full = bar_q + 8;
  const uint32_t bar_k_empty = bar_k_full + 8 * KST;
  const uint32_t bar_v_full = bar_k_empty + 8 * KST;
  const uint32_t bar_v_empty = bar_v_full + 8 * VST;
  const uint32_t bar_s_full = bar_v_empty + 8 * VST;  // QK(j) done
  const uint32_t bar_s_free = bar_s_full + 8;          // softmax has read S(j)
  const uint32_t bar_p_full = bar_s_free + 8;          // P(j) written
  const uint32_t bar_o_full = bar_p_full + 8;          // PV(j) done
  const uint32_t bar_o_done = bar_o_full + 8;          // after the last PV
  const uint32_t bar_drain = bar_o_done + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(bar_k_full + 8 * s, 1);
      mbar_init(bar_k_empty + 8 * s, 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(bar_v_full + 8 * s, 1);
      mbar_init(bar_v_empty + 8 * s, 1);
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 128);
    mbar_init(bar_p_full, 128);
    mbar_init(bar_o_full, 1);
    mbar_init(bar_o_done, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_q);
  }
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
      // in-flight loads, for the drain on abort: bit s of k_bits / v_bits,
      // with the phase parity they complete
      uint32_t k_bits = 0, k_par = 0, v_bits = 0, v_par = 0;
      mbar_arrive_expect_tx(bar_q, Q_BYTES);
      tma_load_2d(sbase + OFF_Q, &tmap_q, bar_q, h * HD, row0 + q0);
      for (int j = 0; j < ntiles; ++j) {
        const int ks = j % KST, vs = j % VST;
        const uint32_t kph = (uint32_t)(j / KST) & 1u, vph = (uint32_t)(j / VST) & 1u;
        if (!mbar_wait(bar_k_empty + 8 * ks, kph ^ 1, abort_flag, args.err, kDevErrTimeoutAttn))
          break;
        mbar_arrive_expect_tx(bar_k_full + 8 * ks, KV_TILE);
        tma_load_2d(sbase + OFF_K + ks * KV_TILE, &tmap_q, bar_k_full + 8 * ks, dim + h * HD,
                    row0 + j * BKV);
        k_bits |= 1u << ks;
        k_par = (k_par & ~(1u << ks)) | (kph << ks);
        if (!mbar_wait(bar_v_empty + 8 * vs, vph ^ 1, abort_flag, args.err, kDevErrTimeoutAttn))
          break;
        mbar_arrive_expect_tx(bar_v_full + 8 * vs, KV_TILE);
        tma_load_2d(sbase + OFF_V + vs * KV_TILE, &tmap_q, bar_v_full + 8 * vs,
                    2 * dim + h * HD, row0 + j * BKV);
        v_bits |= 1u << vs;
        v_par = (v_par & ~(1u << vs)) | (vph << vs);
      }
      if (*abort_flag) {
        mbar_wait_drain(bar_q, 0);
        for (int s = 0; s < KST; ++s)
          if (k_bits & (1u << s)) mbar_wait_drain(bar_k_full + 8 * s, (k_par >> s) & 1u);
        for (int s = 0; s < VST; ++s)
          if (v_bits & (1u << s)) mbar_wait_drain(bar_v_full + 8 * s, (v_par >> s) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    // S is double-buffered through the softmax threads' registers: the
    // softmax releases S(j) as soon as it has loaded it, so Q K^T of tile
    // j+2 is issued right after PV(j), a full key tile ahead of its use.
    if (lane == 0) {
      bool issued_any = false, ok = true;
      const uint64_t dq = umma_desc_sw128(sbase + OFF_Q);
      auto issue_qk = [&](int j) {
        const uint64_t dk = umma_desc_sw128(sbase + OFF_K + (j % KST) * KV_TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16_ss(tmem + COL_S, desc_advance(dq, kk * 32), desc_advance(dk, kk * 32),
                      IDESC_S, kk != 0);
        umma_commit(bar_s_full);
        umma_commit(bar_k_empty + 8 * (j % KST));
        issued_any = true;
      };
      auto issue_pv = [&](int j) {
        const uint64_t dv = umma_desc_sw128_mn(sbase + OFF_V + (j % VST) * KV_TILE);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_f16_ts(tmem + COL_O, tmem + COL_P + kk * 8, desc_advance(dv, kk * 2048),
                      IDESC_O, (j | kk) != 0);
        umma_commit(bar_o_full);
        umma_commit(bar_v_empty + 8 * (j % VST));
      };
      auto wait = [&](uint32_t bar, uint32_t ph) {
        return mbar_wait(bar, ph, abort_flag, args.err, kDevErrTimeoutAttn);
      };
      auto wait_k = [&](int j) {
        return wait(bar_k_full + 8 * (j % KST), (uint32_t)(j / KST) & 1u);
      };
      ok = wait(bar_q, 0) && wait_k(0);
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      if (ok && ntiles > 1) {
        ok = wait_k(1) && wait(bar_s_free, 0);
        if (ok) {
          tc_fence_after();
          issue_qk(1);
        }
      }
      for (int j = 0; j < ntiles && ok; ++j) {
        ok = wait(bar_p_full, (uint32_t)j & 1u) &&
             wait(bar_v_full + 8 * (j % VST), (uint32_t)(j / VST) & 1u);
        if (!ok) break;
        tc_fence_after();
        issue_pv(j);
        if (j + 2 < ntiles) {
          ok = wait_k(j + 2) && wait(bar_s_free, (uint32_t)(j + 1) & 1u);
          if (!ok) break;
          tc_fence_after();
          issue_qk(j + 2);
        }
      }
      if (ok) umma_commit(bar_o_done);
      if (*abort_flag && issued_any) {
        umma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------- softmax rows
    constexpr float kRescaleLog2 = 8.0f;
    const int quad = warp & 3;      // this warp's TMEM lane quadrant
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t s_col = lane_base + COL_S;
    const uint32_t p_col = lane_base + COL_P;
    const uint32_t o_col = lane_base + COL_O;
    const float c = args.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    griddep_wait();  // before this grid's output rows are written
    for (int j = 0; j < ntiles && ok; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full, (uint32_t)j & 1u, abort_flag,
                                             args.err, kDevErrTimeoutAttn));
      if (!ok) break;
      tc_fence_after();
      // The scores in two halves: the maximum of the first 64 runs while the
      // second 64 are still on their way from tensor memory.
      uint32_t v[BKV];
      const int valid = min(BKV, seq - j * BKV);  // only the last tile can be ragged
      float mx[4];
      auto half_max = [&](int q0) {
        if (valid < BKV) {
#pragma unroll
          for (int e = 0; e < BKV / 2; ++e)
            if (q0 * 32 + e >= valid) v[q0 * 32 + e] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int q = q0; q < q0 + 2; ++q) {
          float m = fmaxf(__uint_as_float(v[32 * q]), __uint_as_float(v[32 * q + 31]));
#pragma unroll
          for (int e = 1; e < 31; e += 2)
            m = max3f(m, __uint_as_float(v[32 * q + e]), __uint_as_float(v[32 * q + e + 1]));
          mx[q] = m;
        }
      };
      tmem_ld_32x32b_x32(s_col, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_32x32b_x32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_wait_ld();
      tmem_ld_32x32b_x32(s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(v + 64));
      tmem_ld_32x32b_x32(s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(v + 96));
      half_max(0);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar_s_free);  // the next Q K^T may overwrite S now
      half_max(2);
      const float m_tile = max3f(fmaxf(mx[0], mx[1]), mx[2], mx[3]) * c;
      const bool grow = m_tile > m_run + kRescaleLog2;
      const float m_use = grow ? m_tile : m_run;
      const float alpha = grow ? ex2_approx(m_run - m_use) : 1.0f;  // 0 on the first tile
      // All 128 exponentials into registers first (the packed pairs take the
      // scores' registers), so PV(j-1), which still reads P and O, completes
      // under them; only the stores wait for it.
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[BKV / 2];
#pragma unroll
      for (int e = 0; e < BKV / 2; ++e) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(v[2 * e]), c, -m_use));
        const float p1 = ex2_approx(fmaf(__uint_as_float(v[2 * e + 1]), c, -m_use));
        ls[e & 3] += p0 + p1;
        pk[e] = pack_half2(p0, p1);
      }
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o_full, (uint32_t)(j - 1) & 1u, abort_flag,
                                               args.err, kDevErrTimeoutAttn));
        if (!ok) break;
        tc_fence_after();
      }
#pragma unroll
      for (int cc = 0; cc < BKV / 32; ++cc)
        tmem_st_32x32b_x16(p_col + cc * 16, *reinterpret_cast<uint32_t(*)[16]>(pk + 16 * cc));
      const float l_tile = (ls[0] + ls[1]) + (ls[2] + ls[3]);
      l_run = fmaf(l_run, alpha, l_tile);
      m_run = m_use;
      // The rescale uses warp-collective tcgen05.ld/st, so the whole warp takes
      // the branch when any of its rows grew (alpha is 1 for the others).
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        uint32_t o[HD];
        tmem_ld_32x32b_x32(o_col, *reinterpret_cast<uint32_t(*)[32]>(o));
        tmem_ld_32x32b_x32(o_col + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
        tmem_wait_ld();
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * alpha);
#pragma unroll
        for (int q = 0; q < HD / 16; ++q)
          tmem_st_32x32b_x16(o_col + q * 16, *reinterpret_cast<uint32_t(*)[16]>(o + 16 * q));
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p_full);
    }
    if (ok)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar_o_done, 0u, abort_flag, args.err, kDevErrTimeoutAttn));
    if (ok) {
      tc_fence_after();
      uint32_t o[HD];
      tmem_ld_32x32b_x32(o_col, *reinterpret_cast<uint32_t(*)[32]>(o));
      tmem_ld_32x32b_x32(o_col + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
      tmem_wait_ld();
      const int q = q0 + r;
      if (q < seq) {
        const float inv = 1.f / l_run;
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

// Global attention with 128-key tiles over `batch * groups` row ranges of
// `seq` rows each (see attention_tc for the row mapping).
sam3_status_t attention_pp(sam3_ctx_t* ctx, const uint16_t* qkv, int batch, int seq, int heads,
                           float scale, uint16_t* o, int groups, int img_rows, int first_row) {
  const int dim = heads * HD;
  CUtensorMap map_q;
  cuuint64_t dims[2] = {(cuuint64_t)(3 * dim), (cuuint64_t)batch * img_rows};
  cuuint64_t strides[1] = {(cuuint64_t)(3 * dim) * 2};
  cuuint32_t box[2] = {HD, BQ};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_tiled()(&map_q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                              const_cast<uint16_t*>(qkv), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, SAM3_ERR_CUDA, "attention: cuTensorMapEncodeTiled (Q) failed (%d)", (int)r);
  const sam3_status_t st =
      ensure_smem_attr(ctx, kSmemAttnPP, attn_pp_kernel, SMEM_BYTES, "attention smem attribute");
  if (st != SAM3_OK) return st;
  PPArgs a;
  a.out = reinterpret_cast<__half*>(o);
  a.err = ctx->dev_err;
  a.seq = seq;
  a.groups = groups;
  a.img_rows = img_rows;
  a.first_row = first_row;
  a.heads = heads;
  a.dim = dim;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.o32 = (reinterpret_cast<uintptr_t>(o) & 31u) == 0;
  dim3 grid((seq + BQ - 1) / BQ, heads, batch * groups);
  const cudaError_t e = launch_pdl(attn_pp_kernel, grid, dim3(THREADS), SMEM_BYTES, ctx->stream,
                                   map_q, a);
  return check_launch_ret(ctx, e, "attn_pp_kernel");
}

}  // namespace sam3
