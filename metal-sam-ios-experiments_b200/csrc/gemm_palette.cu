// gemm_palette.cu - uint8-palette dequantization fused into an sm_100a
// tcgen05 GEMM:  Y[m, n] = epilogue( X[m, :] . W[n, :] + b[n] ),
// W[n, k] = P[n, idx[n, k]] with one 256-entry fp16 palette per output row.
//
// Reference path replaced: the dense-fp16 MPSGraph matrixMultiplication calls
// of MPSAttention.swift:113-117,179-183 and ViTEncoder.swift:979-997, fed by
// the never-dispatched LUT expansion of Metal/Dequantize.metal:17-93. Here the
// LUT expansion happens in shared memory right before the tensor cores read
// the tile: no dequantized weight is ever written to HBM.
//
// Kernel structure (one persistent CTA per SM, 320 threads):
//   warp 0      TMA producer: X tile [128 x 64] fp16 (128B swizzle) and the
//               uint8 index tile [128 x 64] (64B swizzle) per k-block stage.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M=128, N=128, K=16 per instruction, fp32 accumulators in two
//               128-column TMEM buffers so the epilogue overlaps the next tile).
//   warps 2-5   palette expanders: thread r owns weight row r of the tile;
//               its palette sits in shared memory transposed as 32-bit words
//               word[e & 127][r] = P[r][e & 127] | P[r][(e & 127) + 128] << 16,
//               so lane r always reads bank r (conflict-free lookups), and the
//               fp16 row is written straight into the 128B-swizzled K-major
//               operand layout the UMMA descriptor expects.
//   warps 6-9   epilogue: tcgen05.ld 32 columns at a time, bias / exact GELU /
//               2D-RoPE on the q,k thirds / residual add, fp16 store.
// A dense-fp16-weight variant (TMA-loaded B, used by the patch embedding)
// shares the kernel.
#include "common.cuh"
#include "internal.h"

namespace sam3 {
namespace {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4;
constexpr int NUM_THREADS = 320;
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int B_STAGE = BN * BK * 2;  // 16 KB
constexpr int I_STAGE = BN * BK;      // 8 KB
constexpr int PAL_BYTES = BN * 512;   // 64 KB
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
constexpr int OFF_I = OFF_B + STAGES * B_STAGE;
constexpr int OFF_P = OFF_I + STAGES * I_STAGE;
constexpr int OFF_BAR = OFF_P + PAL_BYTES;
constexpr int NUM_BARS = 3 * STAGES + 6;
constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + slack for 1024-B alignment
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = umma_idesc_f16(BM, BN);
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

enum BMode { kPalette = 0, kDense = 1 };

struct GemmArgs {
  const __half* bias;
  const __half* residual;
  const float* rope;
  // Axial RoPE: when set, rope points at the axial table of rope_rows
  // coordinates, pair-major: float4 element q * rope_rows + c holds the
  // (cos, sin) of pairs 2q and 2q+1 at coordinate c; row r of the output
  // takes its coordinates from rope_pos[r] = x | y << 16 (pairs 0-15 of a head
  // rotate by x, pairs 16-31 by y; -1: no rotation). Otherwise rope is a
  // table of rope_rows full rows (32 pairs) indexed by r % rope_rows.
  const int32_t* rope_pos;
  const __half* palette;
  __half* y;
  int* err;
  int m, n, k;
  int epi;
  int rope_rows;
  int qk_cols;
  int m_tiles, total_tiles;
  int y32;    // y is 32-byte aligned: 256-bit stores
  int res32;  // residual is 32-byte aligned: 256-bit loads
};


// f[0..7] += the 8 fp16 values of v (packed fp32x2 adds).
__device__ __forceinline__ void add_half8(float* f, uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 s = __fadd2_rn(make_float2(f[2 * q], f[2 * q + 1]), unpack_half2(w[q]));
    f[2 * q] = s.x;
    f[2 * q + 1] = s.y;
  }
}

__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Coordinates of an output row for the axial RoPE epilogue (loaded before
// the accumulator is ready).
__device__ __forceinline__ int rope_pos_of(const GemmArgs& a, int row) {
  return (a.rope_pos && a.epi == SAM3_EPI_BIAS_ROPE_QKV && row < a.m) ? __ldg(a.rope_pos + row)
                                                                       : 0;
}

// Warm L1 with an epilogue's inputs for 64 columns of one output row (bias,
// RoPE table row, residual row) while the accumulator is still being computed.
// (The axial RoPE table is a few KB and stays in L1 by itself.)
__device__ __forceinline__ void epilogue_prefetch(const GemmArgs& a, int row, int col0) {
  if (a.bias) prefetch_l1(a.bias + col0);
  if (a.epi == SAM3_EPI_BIAS_ROPE_QKV && col0 < a.qk_cols && !a.rope_pos) {
    const float* t = a.rope + (size_t)(row % a.rope_rows) * 64;
    prefetch_l1(t);
    prefetch_l1(t + 32);
  }
  if (a.epi == SAM3_EPI_BIAS_RESIDUAL && row < a.m)
    prefetch_l1(a.residual + (size_t)row * a.n + col0);
}

// Epilogue for 32 consecutive accumulator columns of one output row.
// res: the chunk's 32 residual values (4 x 16 bytes) already in registers,
// or null to load them here.
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int row, int col0,
                                               const uint32_t (&v)[32], int rpos,
                                               const uint4* res = nullptr) {
  float f[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
  if (a.bias) {
    const uint4* bp = reinterpret_cast<const uint4*>(a.bias + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) add_half8(f + 8 * q, __ldg(bp + q));
  }
  if (a.epi == SAM3_EPI_BIAS_GELU) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float2 g = gelu_as2(make_float2(f[j], f[j + 1]));
      f[j] = g.x;
      f[j + 1] = g.y;
    }
  } else if (a.epi == SAM3_EPI_BIAS_ROPE_QKV && col0 < a.qk_cols) {
    // 32 columns = 16 interleaved (even, odd) pairs of one 64-wide head;
    // a full table row holds 32 (cos, sin) pairs, pair j at float offset 2j;
    // the axial table holds the 16 pairs of one coordinate (x for the first
    // 32 columns of the head, y for the last 32), pair-major: the float4 of
    // pairs (2q, 2q+1) at coordinate c is element q * rope_rows + c, so the
    // 32 lanes of a warp (32 consecutive tokens, consecutive x) read
    // consecutive 16-byte entries instead of 32 different cache lines.
    const float4* t;
    int tstride = 1;
    bool rotate = true;
    if (a.rope_pos) {
      rotate = rpos >= 0;
      const int c = (col0 & 32) ? (rpos >> 16) : (rpos & 0xFFFF);
      t = reinterpret_cast<const float4*>(a.rope) + (rotate ? c : 0);
      tstride = a.rope_rows;
    } else {
      t = reinterpret_cast<const float4*>(a.rope + (size_t)(row % a.rope_rows) * 64 + (col0 & 63));
    }
#pragma unroll
    for (int q = 0; q < 8 && rotate; ++q) {
      const float4 cs = __ldg(t + q * tstride);
      float x0 = f[4 * q], x1 = f[4 * q + 1];
      f[4 * q] = x0 * cs.x - x1 * cs.y;
      f[4 * q + 1] = x0 * cs.y + x1 * cs.x;
      x0 = f[4 * q + 2];
      x1 = f[4 * q + 3];
      f[4 * q + 2] = x0 * cs.z - x1 * cs.w;
      f[4 * q + 3] = x0 * cs.w + x1 * cs.z;
    }
  }
  if (row >= a.m) return;
  const size_t off = (size_t)row * a.n + col0;
  if (a.epi == SAM3_EPI_BIAS_RESIDUAL) {
    uint4 r[4];
    if (res) {
#pragma unroll
      for (int q = 0; q < 4; ++q) r[q] = res[q];
    } else if (a.res32) {
      ld_global_v8(a.residual + off, r[0], r[1]);
      ld_global_v8(a.residual + off + 16, r[2], r[3]);
    } else {
      const uint4* rp = reinterpret_cast<const uint4*>(a.residual + off);
#pragma unroll
      for (int q = 0; q < 4; ++q) r[q] = rp[q];
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) add_half8(f + 8 * q, r[q]);
  }
  // Each lane writes its own row: 32-byte stores fill whole sectors and halve
  // the store instructions (the epilogue's issue cost slows the whole GEMM).
  if (a.y32) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = pack_half2(f[16 * h + 2 * e], f[16 * h + 2 * e + 1]);
      st_global_v8(a.y + off + 16 * h, o);
    }
    return;
  }
  uint4* yp = reinterpret_cast<uint4*>(a.y + off);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 o;
    o.x = pack_half2(f[8 * q + 0], f[8 * q + 1]);
    o.y = pack_half2(f[8 * q + 2], f[8 * q + 3]);
    o.z = pack_half2(f[8 * q + 4], f[8 * q + 5]);
    o.w = pack_half2(f[8 * q + 6], f[8 * q + 7]);
    yp[q] = o;
  }
}

// Expand 16 palette indices (one 16-byte idx chunk) of weight row r into 16
// fp16 values = 8 packed words. pal points at word[0][r]; word[e][r] is at
// pal[e * 128].
__device__ __forceinline__ void expand16(uint4 v, const uint32_t* pal, uint32_t (&out)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t u = w[q];
    const uint32_t p0 = pal[(u & 0x7Fu) << 7];
    const uint32_t p1 = pal[((u >> 8) & 0x7Fu) << 7];
    const uint32_t p2 = pal[((u >> 16) & 0x7Fu) << 7];
    const uint32_t p3 = pal[((u >> 24) & 0x7Fu) << 7];
    // bit 7 of each index selects the high half-word (entries 128..255).
    const uint32_t t = (u >> 6) & 0x02020202u;
    const uint32_t sel01 = 0x5410u | ((t & 0x0202u) * 0x11u);
    const uint32_t sel23 = 0x5410u | (((t >> 16) & 0x0202u) * 0x11u);
    out[2 * q] = __byte_perm(p0, p1, sel01);
    out[2 * q + 1] = __byte_perm(p2, p3, sel23);
  }
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_palette_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Round up to 1024 B by offsetting the __shared__ array itself, so every
  // access below stays a shared-memory access (LDS/STS) for the compiler.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t bar_full = sbase + OFF_BAR;
  const uint32_t bar_full_b = bar_full + 8 * STAGES;
  const uint32_t bar_empty = bar_full_b + 8 * STAGES;
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;
  const uint32_t bar_tempty = bar_tfull + 16;
  const uint32_t bar_drain = bar_tempty + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_full_b + 8 * s, 128);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, 128);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int G = gridDim.x;
  const int t_begin = (int)((long long)blockIdx.x * args.total_tiles / G);
  const int t_end = (int)((long long)(blockIdx.x + 1) * args.total_tiles / G);
  const int kblocks = args.k / BK;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issued_par = 0;
      const uint32_t bytes = A_STAGE + (MODE == kPalette ? I_STAGE : B_STAGE);
      for (int t = t_begin; t < t_end; ++t) {
        const int m0 = (t % args.m_tiles) * BM, n0 = (t / args.m_tiles) * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, abort_flag, args.err,
                         kDevErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_full + 8 * s, bytes);
          tma_load_2d(sbase + OFF_A + s * A_STAGE, &tmap_a, bar_full + 8 * s, kb * BK, m0);
          if (MODE == kPalette)
            tma_load_2d(sbase + OFF_I + s * I_STAGE, &tmap_b, bar_full + 8 * s, kb * BK, n0);
          else
            tma_load_2d(sbase + OFF_B + s * B_STAGE, &tmap_b, bar_full + 8 * s, kb * BK, n0);
          issued |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
      }
      if (*abort_flag) {
        // Let every copy this thread issued land before the CTA can exit.
        for (int q = 0; q < STAGES; ++q)
          if (issued & (1u << q)) mbar_wait_drain(bar_full + 8 * q, (issued_par >> q) & 1u);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool issued_any = false;
      for (int t = t_begin; t < t_end; ++t, ++it) {
        const int acc = it & 1;
        const uint32_t use = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(bar_tempty + 8 * acc, use ^ 1, abort_flag, args.err, kDevErrTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar_full + 8 * s, ph, abort_flag, args.err, kDevErrTimeoutMma) ||
              (MODE == kPalette &&
               !mbar_wait(bar_full_b + 8 * s, ph, abort_flag, args.err, kDevErrTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + OFF_A + s * A_STAGE;
          const uint32_t b_addr = sbase + OFF_B + s * B_STAGE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_ss(d_tmem, umma_desc_sw128(a_addr + kk * 32),
                        umma_desc_sw128(b_addr + kk * 32), IDESC, (kb | kk) != 0);
          umma_commit(bar_empty + 8 * s);
          issued_any = true;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(bar_tfull + 8 * acc);
      }
      if (*abort_flag && issued_any) {
        umma_commit(bar_drain);
        mbar_wait_drain(bar_drain, 0);
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------- palette expanders
    // Thread r owns weight row r of the tile: it stages that row's palette,
    // reads only that row's indices and writes only that row of the B tile,
    // so the expanders never need to synchronise with each other.
    if (MODE == kPalette) {
      const int r = threadIdx.x - 64;
      uint32_t* pal = reinterpret_cast<uint32_t*>(smem + OFF_P) + r;  // word[e][r] at pal[e*128]
      int s = 0;
      uint32_t ph = 0;
      int cur_n = -1;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t) {
        const int n_tile = t / args.m_tiles;
        if (n_tile != cur_n) {
          const uint4* prow =
              reinterpret_cast<const uint4*>(args.palette + (size_t)(n_tile * BN + r) * 256);
#pragma unroll 4
          for (int j = 0; j < 16; ++j) {
            const uint4 lo = __ldg(prow + j), hi = __ldg(prow + 16 + j);
            const uint32_t l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int e = 8 * j + 2 * q;
              pal[e * 128] = __byte_perm(l[q], h[q], 0x5410u);
              pal[(e + 1) * 128] = __byte_perm(l[q], h[q], 0x7632u);
            }
          }
          cur_n = n_tile;
        }
        for (int kb = 0; kb < kblocks; ++kb) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_full + 8 * s, ph, abort_flag, args.err,
                                                 kDevErrTimeoutDequant));
          if (!ok) break;
          const uint8_t* itile = smem + OFF_I + s * I_STAGE + r * 64;
          uint8_t* brow = smem + OFF_B + s * B_STAGE + r * 128;
          const int sw64 = (r >> 1) & 3;
          const int sw128 = r & 7;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(itile + ((q ^ sw64) << 4));
            uint32_t o[8];
            expand16(v, pal, o);
            *reinterpret_cast<uint4*>(brow + (((2 * q) ^ sw128) << 4)) =
                make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(brow + (((2 * q + 1) ^ sw128) << 4)) =
                make_uint4(o[4], o[5], o[6], o[7]);
          }
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
          mbar_arrive(bar_full_b + 8 * s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad + 32) belong to this warp
    int it = 0;
    for (int t = t_begin; t < t_end; ++t, ++it) {
      const int acc = it & 1;
      const uint32_t use = (uint32_t)(it >> 1) & 1u;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_tfull + 8 * acc, use, abort_flag,
                                                        args.err, kDevErrTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
      const int m0 = (t % args.m_tiles) * BM, n0 = (t / args.m_tiles) * BN;
      const int row = m0 + quad * 32 + lane;
      const int rpos = rope_pos_of(args, row);
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + (uint32_t)(c * 32), v);
        tmem_wait_ld();
        epilogue_chunk(args, row, n0 + c * 32, v, rpos);
      }
      tc_fence_before();
      mbar_arrive(bar_tempty + 8 * acc);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ============================================================================
// Weight-stationary pair kernel (K <= 1024): a cluster of two CTAs owns a
// 128-row weight slab (64 rows per CTA); each CTA expands its 64 x K slab into
// shared memory ONCE (128 KB fp16, 128B-swizzled K-major, one 8 KB block per
// 64-wide k-block) and then streams every 256-row M tile of its range past it
// with pair MMAs (tcgen05 cta_group::2, M=256, N=128, K=16): the even CTA
// issues, A rows come from both CTAs, B columns from both slabs, and each
// CTA's tensor memory receives its own 128 output rows. Lookups drop from one
// per MAC-row to one per weight per slab, and shared-memory operand traffic is
// 96 B/clk/SM instead of the 1-CTA kernel's 128.
//   warp 0     TMA producer of this CTA's A tiles (6-stage ring); completion
//              is signalled on the even CTA's barrier.
//   warp 1     TMEM allocator (512 columns = 4 accumulators of 128) and, in
//              the even CTA, the MMA issuer.
//   warps 2-9  slab expanders when the N tile changes, epilogue otherwise
//              (two warps per TMEM lane quadrant, 64 columns each).
// ============================================================================
constexpr int WS_BM = 128, WS_BN = 64, WS_BK = 64, WS_KMAX = 1024;
// An A stage holds WS_KSPLIT 64-wide k-blocks (two TMA boxes): the MMA
// issuer then issues 8 pair MMAs per barrier wait. Each mbarrier wait costs
// the single issuing thread far longer than a pair MMA of N=128 takes to
// execute, so 4 MMAs per wait starve the tensor pipe.
constexpr int WS_KSPLIT = 2;
constexpr int WS_A_BOX = WS_BM * WS_BK * 2;           // 16 KB per 64-wide k-block
constexpr int WS_STAGES = 3;
constexpr int WS_A_STAGE = WS_KSPLIT * WS_A_BOX;      // 32 KB
constexpr int WS_SLAB_KB = WS_BN * WS_BK * 2;         // 8 KB per k-block
constexpr int WS_OFF_SLAB = 0;
constexpr int WS_OFF_A = (WS_KMAX / WS_BK) * WS_SLAB_KB;  // 128 KB
constexpr int WS_OFF_PAL = WS_OFF_A;  // palette staging overlays the drained A ring
constexpr int WS_NUM_ACC = 4, WS_ACC_COLS = 128;
constexpr int WS_OFF_BAR = WS_OFF_A + WS_STAGES * WS_A_STAGE;
constexpr int WS_NUM_BARS = 2 * WS_STAGES + 2 * WS_NUM_ACC + 4;
constexpr int WS_OFF_MISC = WS_OFF_BAR + WS_NUM_BARS * 8;
constexpr int WS_SMEM_BYTES = WS_OFF_MISC + 16 + 1024;
constexpr int WS_THREADS = 320;
constexpr int WS_NUM_EXP = 256;  // warps 2-9
constexpr uint32_t WS_TMEM_COLS = 512;
constexpr uint32_t WS_IDESC = umma_idesc_f16(2 * WS_BM, 2 * WS_BN);
static_assert(WS_SMEM_BYTES <= 232448, "shared memory budget");
static_assert(WS_BN * 128 * 4 <= WS_STAGES * WS_A_STAGE, "palette staging fits the A ring");

// Expand weight row `exp_row` (0..63) of this CTA, columns [k0, k0 + 16*N16),
// into a slab buffer laid out as 64-row x 128-byte swizzled blocks per
// 64-wide k-block, k-blocks counted from `kbase`. pal = word[e][r] at
// pal[e*64].
// All N16 16-byte index loads of the range are issued before the first
// lookup, so the thread waits for one L2 round trip instead of N16.
// Per 4 indices: one `prmt` per lookup builds its byte offset
// (index & 127) * 256 + r * 4, and one sign-replicating `prmt` plus one
// `lop3` build the two half-word selectors (bit 7 of an index picks the
// high half of its word).
template <int N16>
__device__ __forceinline__ void ws_expand_loaded(const uint4 (&iv)[N16], const uint32_t* pal,
                                                 uint8_t* buf, int exp_row, int k0, int kbase) {
  const int sw = exp_row & 7;
  const uint8_t* palb = reinterpret_cast<const uint8_t*>(pal - exp_row);
  const uint32_t rowoff = (uint32_t)exp_row * 4u;  // < 256: byte 0 only
#pragma unroll
  for (int i = 0; i < N16; ++i) {
    const int k = k0 + 16 * i;
    const uint4 v = iv[i];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t uu = w4[q];
      const uint32_t m = uu & 0x7F7F7F7Fu;
      // offset bytes [r * 4, index j & 127, 0, 0]
      const uint32_t p0 = *reinterpret_cast<const uint32_t*>(palb + __byte_perm(m, rowoff, 0x5504u));
      const uint32_t p1 = *reinterpret_cast<const uint32_t*>(palb + __byte_perm(m, rowoff, 0x5514u));
      const uint32_t p2 = *reinterpret_cast<const uint32_t*>(palb + __byte_perm(m, rowoff, 0x5524u));
      const uint32_t p3 = *reinterpret_cast<const uint32_t*>(palb + __byte_perm(m, rowoff, 0x5534u));
      // selector nibbles 0,1 | 4,5 (low halves), + 2 where the index is >= 128
      const uint32_t sel = (byte_sign_mask(uu) & 0x22222222u) | 0x54105410u;
      o[2 * q] = __byte_perm(p0, p1, sel);
      o[2 * q + 1] = __byte_perm(p2, p3, sel >> 16);
    }
    const int kb = (k - kbase) >> 6, c = (k & 63) >> 3;
    uint8_t* dst = buf + kb * WS_SLAB_KB + exp_row * 128;
    *reinterpret_cast<uint4*>(dst + ((c ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(dst + (((c + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}
template <int N16>
__device__ __forceinline__ void ws_load_idx(const uint8_t* irow, int k0, uint4 (&iv)[N16]) {
#pragma unroll
  for (int i = 0; i < N16; ++i) iv[i] = __ldg(reinterpret_cast<const uint4*>(irow + k0) + i);
}
template <int N16>
__device__ __forceinline__ void ws_expand_range(const uint8_t* irow, const uint32_t* pal,
                                                uint8_t* buf, int exp_row, int k0, int kbase) {
  uint4 iv[N16];
  ws_load_idx<N16>(irow, k0, iv);
  ws_expand_loaded<N16>(iv, pal, buf, exp_row, k0, kbase);
}

struct WsArgs {
  GemmArgs g;
  const uint8_t* idx;
  int kblocks;
  int m_tiles;  // 256-row pair tiles
  int n_tiles;  // n / 128
  int units;    // n_tiles * m_tiles
  int sets;     // > 0: pair p < sets * n_tiles owns N tile p % n_tiles and M tiles
                // p / n_tiles + k * sets below m_a; the pairs after them share the
                // N-major units of M tiles [m_a, m_tiles) in contiguous ranges;
                // 0: pair p owns a contiguous range of N-major units
  int m_a;      // sets > 0: M tiles swept by the sets (the rest go to the extra pairs)
  int a3d;      // 1: the A map is 3-D (one request per A stage), 0: 2-D boxes
};

// Unit k of pair `pair` -> (n_tile, m_tile); false when the pair has no unit k.
__device__ __forceinline__ bool ws_unit(const WsArgs& wa, int pair, int npairs, int k, int& n_tile,
                                        int& m_tile) {
  if (wa.sets > 0) {
    const int set_pairs = wa.sets * wa.n_tiles;
    if (pair < set_pairs) {
      n_tile = pair % wa.n_tiles;
      m_tile = pair / wa.n_tiles + k * wa.sets;
      return m_tile < wa.m_a;
    }
    const int mb = wa.m_tiles - wa.m_a, e = pair - set_pairs, extra = npairs - set_pairs;
    const long long units_b = (long long)mb * wa.n_tiles;
    const int u = (int)(e * units_b / extra) + k;
    if (u >= (int)((e + 1) * units_b / extra)) return false;
    n_tile = u / mb;
    m_tile = wa.m_a + u % mb;
    return true;
  }
  const int u = (int)((long long)pair * wa.units / npairs) + k;
  if (u >= (int)((long long)(pair + 1) * wa.units / npairs)) return false;
  n_tile = u / wa.m_tiles;
  m_tile = u % wa.m_tiles;
  return true;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(WS_THREADS, 1)
    gemm_ws_kernel(const __grid_constant__ CUtensorMap tmap_a, const WsArgs wa) {
  const GemmArgs& args = wa.g;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  const uint32_t bar_a_full = sbase + WS_OFF_BAR;
  const uint32_t bar_a_empty = bar_a_full + 8 * WS_STAGES;
  const uint32_t bar_tfull = bar_a_empty + 8 * WS_STAGES;
  const uint32_t bar_tempty = bar_tfull + 8 * WS_NUM_ACC;
  const uint32_t bar_slab_full = bar_tempty + 8 * WS_NUM_ACC;  // even CTA's copy used
  const uint32_t bar_slab_local = bar_slab_full + 8;
  const uint32_t bar_exp_sync = bar_slab_local + 8;
  const uint32_t bar_drain = bar_exp_sync + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + WS_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + WS_OFF_MISC + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS_STAGES; ++s) {
      mbar_init(bar_a_full + 8 * s, 1);
      mbar_init(bar_a_empty + 8 * s, 1);
    }
    for (int a = 0; a < WS_NUM_ACC; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, 2 * WS_NUM_EXP / 32);  // one arrive per epilogue warp
    }
    mbar_init(bar_slab_full, 2 * WS_NUM_EXP);
    mbar_init(bar_slab_local, WS_NUM_EXP);
    mbar_init(bar_exp_sync, WS_NUM_EXP);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc_cg2(smem_u32(tmem_slot), WS_TMEM_COLS);
    tmem_relinquish_cg2();
  }
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();

  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int kblocks = wa.kblocks;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      griddep_wait();  // X is the previous kernel's output
      const uint64_t policy = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0, gen = 0;
      int cur_n = -1;
      bool ok = true;
      int n_tile, m_tile;
      for (int k = 0; ok && ws_unit(wa, pair, npairs, k, n_tile, m_tile); ++k) {
        if (n_tile != cur_n) {
          // the slab (and the palette staged over this ring) must be done first
          ok = mbar_wait(bar_slab_local, gen & 1u, abort_flag, args.err, kDevErrTimeoutProducer);
          if (!ok) break;
          ++gen;
          cur_n = n_tile;
        }
        const int row = m_tile * 2 * WS_BM + (int)rank * WS_BM;
        for (int ks = 0; ks < kblocks / WS_KSPLIT; ++ks) {
          if (!mbar_wait_cluster(bar_a_empty + 8 * s, ph ^ 1, abort_flag, args.err,
                                 kDevErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(bar_a_full + 8 * s, 2 * WS_A_STAGE);
          if (wa.a3d)
            tma_load_3d_cg2(sbase + WS_OFF_A + s * WS_A_STAGE, &tmap_a,
                            mapa_shared(bar_a_full + 8 * s, 0), 0, row, ks * WS_KSPLIT, policy);
          else
            for (int h = 0; h < WS_KSPLIT; ++h)
              tma_load_2d_cg2(sbase + WS_OFF_A + s * WS_A_STAGE + h * WS_A_BOX, &tmap_a,
                              mapa_shared(bar_a_full + 8 * s, 0), (ks * WS_KSPLIT + h) * WS_BK,
                              row, policy);
          if (++s == WS_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer (even CTA)
    if (leader && lane == 0) {
      int s = 0, it = 0;
      uint32_t ph = 0, gen = 0;
      int cur_n = -1;
      bool issued_any = false, ok = true;
      int n_tile, m_tile;
      for (int k = 0; ok && ws_unit(wa, pair, npairs, k, n_tile, m_tile); ++k, ++it) {
        if (n_tile != cur_n) {
          ok = mbar_wait_cluster(bar_slab_full, gen & 1u, abort_flag, args.err, kDevErrTimeoutMma);
          if (!ok) break;
          ++gen;
          cur_n = n_tile;
        }
        const int acc = it % WS_NUM_ACC;
        const uint32_t use = (uint32_t)(it / WS_NUM_ACC) & 1u;
        if (!mbar_wait_cluster(bar_tempty + 8 * acc, use ^ 1, abort_flag, args.err,
                               kDevErrTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(acc * WS_ACC_COLS);
        for (int ks = 0; ks < kblocks / WS_KSPLIT; ++ks) {
          if (!mbar_wait_cluster(bar_a_full + 8 * s, ph, abort_flag, args.err, kDevErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(sbase + WS_OFF_A + s * WS_A_STAGE);
          const uint64_t db = umma_desc_sw128(sbase + WS_OFF_SLAB + ks * WS_KSPLIT * WS_SLAB_KB);
#pragma unroll
          for (int h = 0; h < WS_KSPLIT; ++h) {
#pragma unroll
            for (int kk = 0; kk < WS_BK / 16; ++kk)
              umma_f16_ss_cg2(d_tmem, desc_advance(da, h * WS_A_BOX + kk * 32),
                              desc_advance(db, h * WS_SLAB_KB + kk * 32), WS_IDESC,
                              (ks | h | kk) != 0);
          }
          umma_commit_cg2_mc(bar_a_empty + 8 * s, 0x3);
          issued_any = true;
          if (++s == WS_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_cg2_mc(bar_tfull + 8 * acc, 0x3);
      }
      if (*abort_flag && issued_any) {
        umma_commit_cg2(bar_drain);
        mbar_wait_cluster_drain(bar_drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------- expanders + epilogue
    const int ew = warp - 2;                     // 0..7
    const int exp_row = lane + 32 * (ew & 1);    // slab row 0..63
    const int exp_q = ew >> 1;                   // k quarter 0..3
    const int quad = warp & 3;                   // TMEM lane quadrant of this warp
    const int colhalf = ew >> 2;                 // accumulator columns [64*colhalf, +64)
    uint32_t sync_ph = 0;
    int cur_n = -1, it = 0;
    bool ok = true, dep_waited = false;
    int n_tile, m_tile;
    for (int k = 0; ok && ws_unit(wa, pair, npairs, k, n_tile, m_tile); ++k, ++it) {
      if (n_tile != cur_n) {
        // ---- expand this CTA's 64 x K slab of weight rows (all earlier MMAs
        // are complete: their accumulators were drained by this loop).
        const int wrow = n_tile * 2 * WS_BN + (int)rank * WS_BN + exp_row;
        uint32_t* pal = reinterpret_cast<uint32_t*>(smem + WS_OFF_PAL) + exp_row;  // word[e][r] at pal[e*64]
        {
          const uint4* prow = reinterpret_cast<const uint4*>(args.palette + (size_t)wrow * 256);
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // entries [exp_q*32 + 8j, +8) and +128
            const uint4 lo = __ldg(prow + exp_q * 4 + j), hi = __ldg(prow + 16 + exp_q * 4 + j);
            const uint32_t l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int e = exp_q * 32 + 8 * j + 2 * q;
              pal[e * 64] = __byte_perm(l[q], h[q], 0x5410u);
              pal[(e + 1) * 64] = __byte_perm(l[q], h[q], 0x7632u);
            }
          }
        }
        mbar_arrive(bar_exp_sync);
        ok = __all_sync(0xffffffffu, mbar_wait(bar_exp_sync, sync_ph, abort_flag, args.err,
                                               kDevErrTimeoutDequant));
        sync_ph ^= 1;
        if (!ok) break;
        const int kq = args.k / 4;
        const uint8_t* irow = wa.idx + (size_t)wrow * args.k;
        // 128 indices per batch of loads (one L2 round trip), 32 for the rest
        int k = exp_q * kq;
        for (; k + 128 <= (exp_q + 1) * kq; k += 128)
          ws_expand_range<8>(irow, pal, smem + WS_OFF_SLAB, exp_row, k, 0);
        for (; k < (exp_q + 1) * kq; k += 32)
          ws_expand_range<2>(irow, pal, smem + WS_OFF_SLAB, exp_row, k, 0);
        fence_proxy_async_smem();
        mbar_arrive(bar_slab_local);
        mbar_arrive_cluster(mapa_shared(bar_slab_full, 0));
        cur_n = n_tile;
      }
      // ---- epilogue of unit u: its 64 columns of this row go from tensor
      // memory to registers, the accumulator goes straight back to the MMA
      // issuer, then bias / GELU / RoPE / residual and the stores.
      const int acc = it % WS_NUM_ACC;
      const uint32_t use = (uint32_t)(it / WS_NUM_ACC) & 1u;
      const int row = m_tile * 2 * WS_BM + (int)rank * WS_BM + quad * 32 + lane;
      const int col0 = n_tile * 2 * WS_BN + colhalf * 64;
      if (!dep_waited) {  // the slab is weights only; the residual is not
        griddep_wait();
        dep_waited = true;
      }
      epilogue_prefetch(args, row, col0);
      const int rpos = rope_pos_of(args, row);
      // The residual row's 64 values go straight to registers while the
      // accumulator is computed: 256 threads' lines (32 KB) would not stay in
      // the L1 left beside this kernel's shared memory.
      uint4 res[8];
      const bool has_res = args.epi == SAM3_EPI_BIAS_RESIDUAL && row < args.m;
      if (has_res) {
        const __half* rp = args.residual + (size_t)row * args.n + col0;
        if (args.res32) {
#pragma unroll
          for (int q = 0; q < 4; ++q) ld_global_v8(rp + 16 * q, res[2 * q], res[2 * q + 1]);
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) res[q] = reinterpret_cast<const uint4*>(rp)[q];
        }
      }
      ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar_tfull + 8 * acc, use, abort_flag,
                                                     args.err, kDevErrTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) +
                             (uint32_t)(acc * WS_ACC_COLS + colhalf * 64);
      uint32_t v[64];
      tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_32x32b_x32(taddr + 32u, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
      epilogue_chunk(args, row, col0, *reinterpret_cast<const uint32_t(*)[32]>(v), rpos,
                     has_res ? res : nullptr);
      epilogue_chunk(args, row, col0 + 32, *reinterpret_cast<const uint32_t(*)[32]>(v + 32), rpos,
                     has_res ? res + 4 : nullptr);
    }
  }

  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while its pair may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_cg2(tmem, WS_TMEM_COLS);
  }
}

// ============================================================================
// Chunked weight-stationary pair kernel (K > 1024, K % 128 == 0; fc2 with
// K = 4096, or 4736 for the checkpoint): the pair's 128-row slab is expanded
// one 384-wide K chunk at a time (the last one shorter when K % 384 != 0)
// into two alternating 48 KB shared-memory buffers, so the expansion of chunk
// c+1 overlaps the MMAs on chunk c. 384 rather than 512: the 32 KB this frees
// holds a third 32 KB stage of X, and with two stages the MMAs waited for X
// (fc2 782 -> 825 TFLOP/s at M = 82944; 256-wide chunks with four stages ran
// 752, paying more per-chunk barrier round trips). Each expanded chunk feeds a group of two
// 256-row M tiles accumulating in their own TMEM buffers (4 x 128 columns:
// groups alternate between accumulator pairs, so the epilogue of one group,
// run by four epilogue warps of its own, overlaps the next group's MMAs).
// Each pair keeps one N tile (palette staged once, 32 KB); the pairs of a
// "set" share one contiguous range of M tiles, the ranges of the sets
// differing by at most one tile, taken two at a time (the last group of a
// range may hold one). Interleaving whole groups over the sets instead left
// up to a quarter of the pairs idle in the last round (81 groups over 18
// sets at M = 41472).
// ============================================================================
constexpr int WSC_KC = 384;
constexpr int WSC_KB_PER_CHUNK = WSC_KC / WS_BK;                    // 6
constexpr int WSC_BUF = WSC_KB_PER_CHUNK * WS_SLAB_KB;              // 48 KB
constexpr int WSC_STAGES = 3;                                      // A stages of WS_KSPLIT k-blocks
constexpr int WSC_GROUP = 2;                                        // M tiles per group
constexpr int WSC_OFF_SLAB = 0;                                     // 2 buffers
constexpr int WSC_OFF_PAL = 2 * WSC_BUF;                            // 96 KB
constexpr int WSC_OFF_A = WSC_OFF_PAL + WS_BN * 128 * 4;            // 128 KB
constexpr int WSC_OFF_BAR = WSC_OFF_A + WSC_STAGES * WS_A_STAGE;    // 224 KB
constexpr int WSC_NUM_BARS = 2 * WSC_STAGES + 2 + 2 + 2 + 2 + 2;
constexpr int WSC_OFF_MISC = WSC_OFF_BAR + WSC_NUM_BARS * 8;
constexpr int WSC_SMEM_BYTES = WSC_OFF_MISC + 16 + 1024;
static_assert(WSC_SMEM_BYTES <= 232448, "shared memory budget");
// Warps 0 (producer), 1 (MMA issuer), 2-9 (slab expanders) and 10-13, four
// epilogue warps of their own (one per TMEM lane quadrant, all 128 columns of
// a row each): with the epilogue on the expander warps, the MMA issuer waited
// for expanded chunks 24 % of its time (clock64 accounting at M = 82944).
constexpr int WSC_THREADS = 448;
constexpr int WSC_NUM_EPI_WARPS = 4;

struct WscArgs {
  GemmArgs g;
  const uint8_t* idx;
  int chunks;   // ceil(K / 512); the last chunk may hold fewer k-blocks
  int kblocks;  // K / 64 (even)
  int m_tiles;  // 256-row pair tiles
  int n_tiles;  // n / 128
  int sets;     // pairs / n_tiles, at most m_tiles
  int a3d;      // as WsArgs::a3d
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(WSC_THREADS, 1)
    gemm_wsc_kernel(const __grid_constant__ CUtensorMap tmap_a, const WscArgs wa) {
  const GemmArgs& args = wa.g;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  const uint32_t bar_a_full = sbase + WSC_OFF_BAR;
  const uint32_t bar_a_empty = bar_a_full + 8 * WSC_STAGES;
  const uint32_t bar_slab_full = bar_a_empty + 8 * WSC_STAGES;  // [2], even CTA's copy used
  const uint32_t bar_slab_empty = bar_slab_full + 16;           // [2], per CTA (multicast)
  const uint32_t bar_tfull = bar_slab_empty + 16;               // [2] accumulator pairs
  const uint32_t bar_tempty = bar_tfull + 16;                   // [2], even CTA's copy used
  const uint32_t bar_pal = bar_tempty + 16;
  const uint32_t bar_drain = bar_pal + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + WSC_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + WSC_OFF_MISC + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < WSC_STAGES; ++s) {
      mbar_init(bar_a_full + 8 * s, 1);
      mbar_init(bar_a_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_slab_full + 8 * b, 2 * WS_NUM_EXP);
      mbar_init(bar_slab_empty + 8 * b, 1);
      mbar_init(bar_tfull + 8 * b, 1);
      mbar_init(bar_tempty + 8 * b, 2 * WSC_NUM_EPI_WARPS);  // one arrive per epilogue warp
    }
    mbar_init(bar_pal, WS_NUM_EXP);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc_cg2(smem_u32(tmem_slot), WS_TMEM_COLS);
    tmem_relinquish_cg2();
  }
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch_dependents();

  // Pair p owns N tile p % n_tiles and set p / n_tiles's M tiles
  // [m_lo, m_hi): the n_tiles pairs of a set sweep the same A rows together
  // (one DRAM read, the other N tiles hit L2) and each pair stages its
  // palette once. Groups are WSC_GROUP tiles from m_lo; the last may be short.
  const int pair = blockIdx.x >> 1;
  const int my_n = pair % wa.n_tiles, my_set = pair / wa.n_tiles;
  const int m_lo = (int)((long long)my_set * wa.m_tiles / wa.sets);
  const int m_hi = (int)((long long)(my_set + 1) * wa.m_tiles / wa.sets);
  const int chunks = wa.chunks;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      griddep_wait();  // X is the previous kernel's output
      const uint64_t policy = l2_policy_evict_last();
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int mt = m_lo; mt < m_hi && ok; mt += WSC_GROUP) {
        const int gs = min(WSC_GROUP, m_hi - mt);
        for (int c = 0; c < chunks && ok; ++c)
          for (int t = 0; t < gs && ok; ++t) {
            const int row = (mt + t) * 2 * WS_BM + (int)rank * WS_BM;
            const int steps = min(WSC_KB_PER_CHUNK, wa.kblocks - c * WSC_KB_PER_CHUNK) / WS_KSPLIT;
            for (int ks = 0; ks < steps; ++ks) {
              if (!mbar_wait_cluster(bar_a_empty + 8 * s, ph ^ 1, abort_flag, args.err,
                                     kDevErrTimeoutProducer)) {
                ok = false;
                break;
              }
              if (leader) mbar_arrive_expect_tx(bar_a_full + 8 * s, 2 * WS_A_STAGE);
              if (wa.a3d)
                tma_load_3d_cg2(sbase + WSC_OFF_A + s * WS_A_STAGE, &tmap_a,
                                mapa_shared(bar_a_full + 8 * s, 0), 0, row,
                                c * WSC_KB_PER_CHUNK + ks * WS_KSPLIT, policy);
              else
                for (int h = 0; h < WS_KSPLIT; ++h)
                  tma_load_2d_cg2(sbase + WSC_OFF_A + s * WS_A_STAGE + h * WS_A_BOX, &tmap_a,
                                  mapa_shared(bar_a_full + 8 * s, 0),
                                  c * WSC_KC + (ks * WS_KSPLIT + h) * WS_BK, row, policy);
              if (++s == WSC_STAGES) {
                s = 0;
                ph ^= 1;
              }
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer (even CTA)
    if (leader && lane == 0) {
      int s = 0, it = 0, q = 0;
      uint32_t ph = 0;
      bool issued_any = false, ok = true;
      for (int mt = m_lo; mt < m_hi && ok; mt += WSC_GROUP, ++it) {
        const int gp = it & 1, gs = min(WSC_GROUP, m_hi - mt);
        if (!mbar_wait_cluster(bar_tempty + 8 * gp, ((uint32_t)(it >> 1) & 1u) ^ 1u, abort_flag,
                               args.err, kDevErrTimeoutMma))
          break;
        tc_fence_after();
        for (int c = 0; c < chunks && ok; ++c, ++q) {
          const int b = q & 1;
          if (!mbar_wait_cluster(bar_slab_full + 8 * b, (uint32_t)(q >> 1) & 1u, abort_flag,
                                 args.err, kDevErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int steps = min(WSC_KB_PER_CHUNK, wa.kblocks - c * WSC_KB_PER_CHUNK) / WS_KSPLIT;
          for (int t = 0; t < gs && ok; ++t) {
            const uint32_t d_tmem = tmem + (uint32_t)((2 * gp + t) * WS_ACC_COLS);
            for (int ks = 0; ks < steps; ++ks) {
              if (!mbar_wait_cluster(bar_a_full + 8 * s, ph, abort_flag, args.err,
                                     kDevErrTimeoutMma)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t da = umma_desc_sw128(sbase + WSC_OFF_A + s * WS_A_STAGE);
              const uint64_t db = umma_desc_sw128(sbase + WSC_OFF_SLAB + b * WSC_BUF +
                                                  ks * WS_KSPLIT * WS_SLAB_KB);
#pragma unroll
              for (int h = 0; h < WS_KSPLIT; ++h) {
#pragma unroll
                for (int kk = 0; kk < WS_BK / 16; ++kk)
                  umma_f16_ss_cg2(d_tmem, desc_advance(da, h * WS_A_BOX + kk * 32),
                                  desc_advance(db, h * WS_SLAB_KB + kk * 32), WS_IDESC,
                                  (c | ks | h | kk) != 0);
              }
              umma_commit_cg2_mc(bar_a_empty + 8 * s, 0x3);
              issued_any = true;
              if (++s == WSC_STAGES) {
                s = 0;
                ph ^= 1;
              }
            }
          }
          if (ok) umma_commit_cg2_mc(bar_slab_empty + 8 * b, 0x3);
        }
        if (!ok) break;
        umma_commit_cg2_mc(bar_tfull + 8 * gp, 0x3);
      }
      if (*abort_flag && issued_any) {
        umma_commit_cg2(bar_drain);
        mbar_wait_cluster_drain(bar_drain, 0);
      }
    }
  } else if (warp >= 2 + WS_NUM_EXP / 32) {
    // ------------------------------------------------------------- epilogue warps
    // Warp w handles TMEM lane quadrant w % 4 (rows quad*32 + lane of the CTA's
    // 128) and all 128 columns, group after group, in the issuer's order.
    const int quad = warp & 3;
    int it = 0;
    bool ok = true;
    griddep_wait();  // the residual is the previous kernel's output
    for (int mt = m_lo; mt < m_hi && ok; mt += WSC_GROUP, ++it) {
      const int gp = it & 1, gs = min(WSC_GROUP, m_hi - mt);
      const int row0 = mt * 2 * WS_BM + (int)rank * WS_BM + quad * 32 + lane;
#pragma unroll
      for (int t = 0; t < WSC_GROUP; ++t)
#pragma unroll
        for (int ch = 0; ch < 2; ++ch)
          if (t < gs) epilogue_prefetch(args, row0 + t * 2 * WS_BM, my_n * 2 * WS_BN + ch * 64);
      const int rpos0 = rope_pos_of(args, row0), rpos1 = rope_pos_of(args, row0 + 2 * WS_BM);
      ok = __all_sync(0xffffffffu,
                      mbar_wait_cluster(bar_tfull + 8 * gp, (uint32_t)(it >> 1) & 1u, abort_flag,
                                        args.err, kDevErrTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int t = 0; t < gs; ++t) {
        const int row = row0 + t * 2 * WS_BM;
        const int rpos = t == 0 ? rpos0 : rpos1;
#pragma unroll 1
        for (int ch = 0; ch < 2; ++ch) {
          const int col0 = my_n * 2 * WS_BN + ch * 64;
          const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) +
                                 (uint32_t)((2 * gp + t) * WS_ACC_COLS + ch * 64);
          uint32_t v[64];
          tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(v));
          tmem_ld_32x32b_x32(taddr + 32u, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
          tmem_wait_ld();
          if (t == gs - 1 && ch == 1) {  // the accumulator pair is free again
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * gp, 0));
          }
          epilogue_chunk(args, row, col0, *reinterpret_cast<const uint32_t(*)[32]>(v), rpos);
          epilogue_chunk(args, row, col0 + 32, *reinterpret_cast<const uint32_t(*)[32]>(v + 32),
                         rpos);
        }
      }
    }
  } else {
    // ------------------------------------------------------------- slab expanders
    const int ew = warp - 2;
    const int exp_row = lane + 32 * (ew & 1);
    const int exp_q = ew >> 1;
    uint32_t* pal = reinterpret_cast<uint32_t*>(smem + WSC_OFF_PAL) + exp_row;
    uint32_t pal_ph = 0;
    int cur_n = -1, q = 0;
    bool ok = true;
    for (int mt = m_lo; mt < m_hi && ok; mt += WSC_GROUP) {
      const int n_tile = my_n;
      const int wrow = n_tile * 2 * WS_BN + (int)rank * WS_BN + exp_row;
      if (n_tile != cur_n) {
        if (cur_n >= 0) {  // every expander is done with the old palette
          mbar_arrive(bar_pal);
          ok = __all_sync(0xffffffffu, mbar_wait(bar_pal, pal_ph, abort_flag, args.err,
                                                 kDevErrTimeoutDequant));
          pal_ph ^= 1;
          if (!ok) break;
        }
        const uint4* prow = reinterpret_cast<const uint4*>(args.palette + (size_t)wrow * 256);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 lo = __ldg(prow + exp_q * 4 + j), hi = __ldg(prow + 16 + exp_q * 4 + j);
          const uint32_t l[4] = {lo.x, lo.y, lo.z, lo.w}, h[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int e = exp_q * 32 + 8 * j + 2 * qq;
            pal[e * 64] = __byte_perm(l[qq], h[qq], 0x5410u);
            pal[(e + 1) * 64] = __byte_perm(l[qq], h[qq], 0x7632u);
          }
        }
        mbar_arrive(bar_pal);
        ok = __all_sync(0xffffffffu, mbar_wait(bar_pal, pal_ph, abort_flag, args.err,
                                               kDevErrTimeoutDequant));
        pal_ph ^= 1;
        if (!ok) break;
        cur_n = n_tile;
      }
      const uint8_t* irow = wa.idx + (size_t)wrow * args.k;
      constexpr int N16 = WSC_KC / 4 / 16;
      auto full = [&](int c) { return (c + 1) * WSC_KB_PER_CHUNK <= wa.kblocks; };
      // Software pipeline: the indices of the next full chunk are loaded into
      // registers before the wait for this chunk's buffer, so their L2 round
      // trip overlaps that wait and this chunk's expansion.
      uint4 iv_next[N16];
      if (full(0)) ws_load_idx<N16>(irow, exp_q * (WSC_KC / 4), iv_next);
      for (int c = 0; c < chunks && ok; ++c, ++q) {
        const int b = q & 1;
        uint4 iv[N16];
#pragma unroll
        for (int i = 0; i < N16; ++i) iv[i] = iv_next[i];
        // the next chunk: c + 1 of this group, or chunk 0 of the pair's next
        // group (same weight rows)
        const int cn = c + 1 < chunks ? c + 1 : (mt + WSC_GROUP < m_hi ? 0 : -1);
        if (cn >= 0 && full(cn))
          ws_load_idx<N16>(irow, cn * WSC_KC + exp_q * (WSC_KC / 4), iv_next);
        if (q >= 2) {
          ok = __all_sync(0xffffffffu,
                          mbar_wait_cluster(bar_slab_empty + 8 * b, (uint32_t)((q >> 1) - 1) & 1u,
                                            abort_flag, args.err, kDevErrTimeoutDequant));
          if (!ok) break;
        }
        const int kb_c = min(WSC_KB_PER_CHUNK, wa.kblocks - c * WSC_KB_PER_CHUNK);
        if (kb_c == WSC_KB_PER_CHUNK) {
          ws_expand_loaded<N16>(iv, pal, smem + WSC_OFF_SLAB + b * WSC_BUF, exp_row,
                                c * WSC_KC + exp_q * (WSC_KC / 4), c * WSC_KC);
        } else {  // short last chunk: kb_c * 16 indices per quarter, 32 at a time
          const int k0 = c * WSC_KC + exp_q * kb_c * 16;
          for (int k = k0; k < k0 + kb_c * 16; k += 32)
            ws_expand_range<2>(irow, pal, smem + WSC_OFF_SLAB + b * WSC_BUF, exp_row, k,
                               c * WSC_KC);
        }
        fence_proxy_async_smem();
        mbar_arrive_cluster(mapa_shared(bar_slab_full + 8 * b, 0));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_cg2(tmem, WS_TMEM_COLS);
  }
}

// Stand-alone LUT expansion, the bit-exact check of the in-GEMM expansion and
// the B200 form of dequantize_int8_optimized (Metal/Dequantize.metal:71-93):
// 8 weight rows per CTA, their palettes staged in shared memory, 16-byte
// index loads and 2 x 16-byte fp16 stores per thread.
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ idx,
                                                      const __half* __restrict__ pal,
                                                      __half* __restrict__ w, int n, int k) {
  __shared__ __align__(16) uint16_t spal[8][256];
  const int row0 = blockIdx.x * 8;
  {
    const int r = threadIdx.x >> 5, c = threadIdx.x & 31;  // 8 rows x 32 uint4
    if (row0 + r < n)
      reinterpret_cast<uint4*>(spal[r])[c] =
          __ldg(reinterpret_cast<const uint4*>(pal + (size_t)(row0 + r) * 256) + c);
  }
  __syncthreads();
  const int cpr = k / 16;  // 16-index chunks per row
  for (int c = threadIdx.x; c < 8 * cpr; c += blockDim.x) {
    const int r = c / cpr, q = c % cpr;
    if (row0 + r >= n) break;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(idx + (size_t)(row0 + r) * k) + q);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u = wv[j];
      o[2 * j] = (uint32_t)spal[r][u & 0xFF] | ((uint32_t)spal[r][(u >> 8) & 0xFF] << 16);
      o[2 * j + 1] = (uint32_t)spal[r][(u >> 16) & 0xFF] | ((uint32_t)spal[r][u >> 24] << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(w + (size_t)(row0 + r) * k) + 2 * q;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

sam3_status_t make_map_2d(sam3_ctx_t* ctx, CUtensorMap* map, CUtensorMapDataType dt,
                          int elem_bytes, const void* base, uint64_t inner, uint64_t outer,
                          uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_tiled()(map, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, SAM3_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SAM3_OK;
}

// X [m, k] as a 3-D tensor (64 columns, m rows, k/64 column blocks) whose
// box {64, 128, WS_KSPLIT} is one A stage of the pair kernels: WS_KSPLIT
// 128-row x 64-column tiles, 128B-swizzled, one after the other in shared
// memory, exactly the layout of WS_KSPLIT 2-D boxes but in one request.
// Returns false when the driver does not accept the map (the kernels then
// issue the 2-D boxes).
bool make_map_a3d(CUtensorMap* map, const void* x, int k, int m) {
  cuuint64_t dims[3] = {(cuuint64_t)WS_BK, (cuuint64_t)m, (cuuint64_t)(k / WS_BK)};
  cuuint64_t strides[2] = {(cuuint64_t)k * 2, (cuuint64_t)WS_BK * 2};
  cuuint32_t box[3] = {(cuuint32_t)WS_BK, (cuuint32_t)WS_BM, (cuuint32_t)WS_KSPLIT};
  cuuint32_t es[3] = {1, 1, 1};
  return encode_tiled()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(x), dims,
                        strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The pairs left over by the sets (max_pairs - sets * n_tiles of them) take
// the last M tiles for every N tile, in contiguous N-major ranges. Returns
// m_a, the M tiles left to the sets: a multiple of `sets` (or all of them)
// that minimises the busier side, counting units (one 256-row M tile by one
// weight slab) for the sets and units plus slab changes for the extra pairs
// (a change drains the MMAs and re-expands a 128 KB slab: about 1.5 units).
int ws_split_m(int m_tiles, int n_tiles, int sets, int max_pairs) {
  const int extra = max_pairs - sets * n_tiles;
  int best = m_tiles;
  long long best_cost = 2LL * ((m_tiles + sets - 1) / sets);
  if (extra <= 0) return best;
  for (int m_a = (m_tiles / sets) * sets; m_a >= sets; m_a -= sets) {
    const int mb = m_tiles - m_a;
    if (mb == 0) continue;
    const long long u = ((long long)mb * n_tiles + extra - 1) / extra;  // per extra pair
    const long long changes = (u + mb - 1) / mb;
    const long long cost = std::max(2LL * (m_a / sets), 2 * u + 3 * changes);
    if (cost < best_cost) {
      best_cost = cost;
      best = m_a;
    }
  }
  return best;
}

sam3_status_t launch_ws(sam3_ctx_t* ctx, const CUtensorMap& ma, const WsArgs& wa) {
  sam3_status_t st = ensure_smem_attr(ctx, kSmemWs, gemm_ws_kernel, WS_SMEM_BYTES,
                                      "gemm_ws smem attribute");
  if (st != SAM3_OK) return st;
  const int max_pairs = ctx->num_sms / 2;
  const int pairs = wa.sets > 0 ? (wa.m_a < wa.m_tiles ? max_pairs : wa.sets * wa.n_tiles)
                                : (wa.units < max_pairs ? wa.units : max_pairs);
  return check_launch_ret(ctx, launch_pdl(gemm_ws_kernel, dim3(2 * pairs), dim3(WS_THREADS),
                                         WS_SMEM_BYTES, ctx->stream, ma, wa),
                          "gemm_ws_kernel");
}

sam3_status_t launch_wsc(sam3_ctx_t* ctx, const CUtensorMap& ma, const WscArgs& wa) {
  sam3_status_t st = ensure_smem_attr(ctx, kSmemWsc, gemm_wsc_kernel, WSC_SMEM_BYTES,
                                      "gemm_wsc smem attribute");
  if (st != SAM3_OK) return st;
  const int pairs = wa.sets * wa.n_tiles;
  return check_launch_ret(ctx, launch_pdl(gemm_wsc_kernel, dim3(2 * pairs), dim3(WSC_THREADS),
                                         WSC_SMEM_BYTES, ctx->stream, ma, wa),
                          "gemm_wsc_kernel");
}

template <int MODE>
sam3_status_t launch(sam3_ctx_t* ctx, const CUtensorMap& ma, const CUtensorMap& mb,
                     const GemmArgs& args) {
  sam3_status_t st = ensure_smem_attr(ctx, kSmemGemm << MODE, gemm_palette_kernel<MODE>,
                                      SMEM_BYTES, "gemm smem attribute");
  if (st != SAM3_OK) return st;
  const int grid = args.total_tiles < ctx->num_sms ? args.total_tiles : ctx->num_sms;
  gemm_palette_kernel<MODE><<<grid, NUM_THREADS, SMEM_BYTES, ctx->stream>>>(ma, mb, args);
  return check_launch(ctx, "gemm_palette_kernel");
}

sam3_status_t validate(sam3_ctx_t* ctx, const void* x, int m, int k, int n, const void* y) {
  if (!x || !y) return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: null x or y");
  if (m <= 0 || n <= 0 || k <= 0)
    return set_error(ctx, SAM3_ERR_SHAPE, "linear: empty shape m=%d n=%d k=%d", m, n, k);
  if (k % BK || n % BN)
    return set_error(ctx, SAM3_ERR_SHAPE, "linear: need k %% 64 == 0 and n %% 128 == 0 (k=%d n=%d)",
                     k, n);
  if (!aligned16(x) || !aligned16(y))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: x and y must be 16-byte aligned");
  return SAM3_OK;
}

}  // namespace

sam3_status_t gemm_palette(sam3_ctx_t* ctx, const uint16_t* x, int m, int k, const uint8_t* idx,
                           const uint16_t* palette, const uint16_t* bias, int n, int epi,
                           const uint16_t* residual, const float* rope, int rope_rows,
                           uint16_t* y, const int32_t* rope_pos) {
  sam3_status_t st = validate(ctx, x, m, k, n, y);
  if (st != SAM3_OK) return st;
  if (!idx || !palette) return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: null idx/palette");
  if (!aligned16(idx) || !aligned16(palette) || (bias && !aligned16(bias)))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: weights must be 16-byte aligned");
  if (epi < SAM3_EPI_BIAS || epi > SAM3_EPI_BIAS_ROPE_QKV)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: bad epilogue %d", epi);
  if (epi == SAM3_EPI_BIAS_RESIDUAL && (!residual || !aligned16(residual)))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: residual epilogue needs aligned residual");
  int qk_cols = 0;
  if (epi == SAM3_EPI_BIAS_ROPE_QKV) {
    if (!rope || (rope_rows <= 0 && !rope_pos) || !aligned16(rope))
      return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: RoPE epilogue needs a table");
    if (n % (3 * 64))
      return set_error(ctx, SAM3_ERR_SHAPE, "linear: RoPE epilogue needs n = 3*heads*64");
    qk_cols = 2 * (n / 3);
  }
  CUtensorMap ma, mb;
  if ((st = make_map_2d(ctx, &ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, (uint64_t)k, (uint64_t)m,
                        BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)) != SAM3_OK)
    return st;
  GemmArgs a;
  a.bias = reinterpret_cast<const __half*>(bias);
  a.residual = reinterpret_cast<const __half*>(residual);
  a.rope = rope;
  a.rope_pos = epi == SAM3_EPI_BIAS_ROPE_QKV ? rope_pos : nullptr;
  a.palette = reinterpret_cast<const __half*>(palette);
  a.y = reinterpret_cast<__half*>(y);
  a.y32 = (reinterpret_cast<uintptr_t>(y) & 31u) == 0;
  a.res32 = (reinterpret_cast<uintptr_t>(a.residual) & 31u) == 0;
  a.err = ctx->dev_err;
  a.m = m;
  a.n = n;
  a.k = k;
  a.epi = epi;
  a.rope_rows = rope_rows > 0 ? rope_rows : 1;
  a.qk_cols = qk_cols;
  a.m_tiles = (m + BM - 1) / BM;
  a.total_tiles = a.m_tiles * (n / BN);
  const double bytes = 2.0 * m * k + 1.0 * n * k + 512.0 * n + 2.0 * m * n *
                       (epi == SAM3_EPI_BIAS_RESIDUAL ? 2 : 1);
  ProfScope prof(ctx, SAM3_PROF_GEMM, 2.0 * m * n * k, bytes);
  if (k <= WS_KMAX && k % (WS_KSPLIT * WS_BK) == 0) {
    // weight-stationary pair kernel: the A map's box is 64 x 128 as above
    WsArgs wa;
    wa.g = a;
    wa.idx = idx;
    wa.kblocks = k / WS_BK;
    wa.m_tiles = (m + 2 * WS_BM - 1) / (2 * WS_BM);
    wa.n_tiles = n / (2 * WS_BN);
    wa.units = wa.m_tiles * wa.n_tiles;
    // Fixed N tile per pair (the pairs of a set sweep M in lockstep, so X is
    // read from DRAM once) when that idles at most 10% of the pairs, or 15%
    // when X is too big to stay in L2 under the contiguous schedule (whose
    // pairs sweep X at 74 different offsets); every pair needs at least two
    // M tiles. Contiguous N-major ranges otherwise.
    const int max_pairs = ctx->num_sms / 2;
    const int sets = wa.n_tiles <= max_pairs ? max_pairs / wa.n_tiles : 0;
    const int idle_pct_limit = 2.0 * m * k > 64.0 * 1024 * 1024 ? 15 : 10;
    wa.sets = (sets > 0 && (max_pairs - sets * wa.n_tiles) * 100 <= idle_pct_limit * max_pairs &&
               wa.m_tiles >= 2 * sets)
                  ? sets
                  : 0;
    wa.m_a = wa.sets > 0 ? ws_split_m(wa.m_tiles, wa.n_tiles, wa.sets, max_pairs) : wa.m_tiles;
    CUtensorMap ma3;
    wa.a3d = make_map_a3d(&ma3, x, k, m) ? 1 : 0;
    return launch_ws(ctx, wa.a3d ? ma3 : ma, wa);
  }
  if (k % (WS_KSPLIT * WS_BK) == 0 && n / (2 * WS_BN) <= ctx->num_sms / 2) {
    // chunked weight-stationary pair kernel (K > 1024; 384-wide chunks, the
    // last one shorter when K % 384 != 0)
    WscArgs wa;
    wa.g = a;
    wa.idx = idx;
    wa.kblocks = k / WS_BK;
    wa.chunks = (k + WSC_KC - 1) / WSC_KC;
    wa.m_tiles = (m + 2 * WS_BM - 1) / (2 * WS_BM);
    wa.n_tiles = n / (2 * WS_BN);
    wa.sets = (ctx->num_sms / 2) / wa.n_tiles;
    if (wa.sets > wa.m_tiles) wa.sets = wa.m_tiles;
    CUtensorMap ma3;
    wa.a3d = make_map_a3d(&ma3, x, k, m) ? 1 : 0;
    return launch_wsc(ctx, wa.a3d ? ma3 : ma, wa);
  }
  if ((st = make_map_2d(ctx, &mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, idx, (uint64_t)k, (uint64_t)n,
                        BK, BN, CU_TENSOR_MAP_SWIZZLE_64B)) != SAM3_OK)
    return st;
  return launch<kPalette>(ctx, ma, mb, a);
}

sam3_status_t gemm_dense(sam3_ctx_t* ctx, const uint16_t* x, int m, int k, const uint16_t* w,
                         const uint16_t* bias, int n, uint16_t* y, int prof_class) {
  sam3_status_t st = validate(ctx, x, m, k, n, y);
  if (st != SAM3_OK) return st;
  if (!w || !aligned16(w) || (bias && !aligned16(bias)))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "dense linear: bad weight pointer");
  CUtensorMap ma, mb;
  if ((st = make_map_2d(ctx, &ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, (uint64_t)k, (uint64_t)m,
                        BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)) != SAM3_OK)
    return st;
  if ((st = make_map_2d(ctx, &mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w, (uint64_t)k, (uint64_t)n,
                        BK, BN, CU_TENSOR_MAP_SWIZZLE_128B)) != SAM3_OK)
    return st;
  GemmArgs a{};
  a.bias = reinterpret_cast<const __half*>(bias);
  a.y = reinterpret_cast<__half*>(y);
  a.y32 = (reinterpret_cast<uintptr_t>(y) & 31u) == 0;
  a.res32 = (reinterpret_cast<uintptr_t>(a.residual) & 31u) == 0;
  a.err = ctx->dev_err;
  a.m = m;
  a.n = n;
  a.k = k;
  a.epi = SAM3_EPI_BIAS;
  a.rope_rows = 1;
  a.m_tiles = (m + BM - 1) / BM;
  a.total_tiles = a.m_tiles * (n / BN);
  ProfScope prof(ctx, prof_class, 2.0 * m * n * k, 2.0 * (m * k + n * k + m * n));
  return launch<kDense>(ctx, ma, mb, a);
}

}  // namespace sam3

using namespace sam3;

extern "C" {

sam3_status_t sam3_linear_palette(sam3_ctx_t* ctx, const uint16_t* x, int32_t m,
                                  const sam3_palette_linear_t* w, int32_t epilogue,
                                  const uint16_t* residual, const float* rope, int32_t rope_rows,
                                  uint16_t* y) {
  SAM3_CHECK_CTX(ctx);
  if (!w) return set_error(ctx, SAM3_ERR_INVALID_ARG, "linear: null weights");
  cudaSetDevice(ctx->device);
  return gemm_palette(ctx, x, m, w->k, w->idx, w->palette, w->bias, w->n, epilogue, residual,
                      rope, rope_rows, y);
}

sam3_status_t sam3_dequant_palette(sam3_ctx_t* ctx, const sam3_palette_linear_t* w,
                                   uint16_t* w_out) {
  SAM3_CHECK_CTX(ctx);
  if (!w || !w->idx || !w->palette || !w_out)
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "dequant: null pointer");
  if (w->n <= 0 || w->k <= 0 || w->k % 16)
    return set_error(ctx, SAM3_ERR_SHAPE, "dequant: need k %% 16 == 0 (n=%d k=%d)", w->n, w->k);
  if (!aligned16(w->idx) || !aligned16(w->palette) || !aligned16(w_out))
    return set_error(ctx, SAM3_ERR_INVALID_ARG, "dequant: pointers must be 16-byte aligned");
  cudaSetDevice(ctx->device);
  ProfScope prof(ctx, SAM3_PROF_OTHER, 0.0, 3.0 * w->n * w->k + 512.0 * w->n);
  dequant_kernel<<<(w->n + 7) / 8, 256, 0, ctx->stream>>>(
      w->idx, reinterpret_cast<const __half*>(w->palette), reinterpret_cast<__half*>(w_out), w->n,
      w->k);
  return check_launch(ctx, "dequant_kernel");
}

}  // extern "C"
