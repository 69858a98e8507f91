// Swap-AB tcgen05 int4 (affine, group 64) verify qmm: y[M,N] = x[M,K] * W[N,K]^T.
//
// Replaces the reference's M=16 verify kernels (dflash_mlx/verify_qmm.py:196-297
// combo_ktmpl, :299-446 super_tree_fp16, :448-547 mma2big, :652-765
// mma2big_pipe) and the stock mx.quantized_matmul(transpose=True) fallback for
// 1 <= M <= 32 rows.  Weight layout is MLX's: w_q uint32 [N, K/8] with nibble
// ki of word p holding column 8p+ki (low nibble first); scales / biases bf16
// [N, K/64]; w = float(nib) * s + b rounded to bf16 (verify_qmm.py:249),
// fp32 accumulation, bf16 output.
//
// Mapping onto Blackwell (M is tiny, so the MMA is "swapped"):
//   * a CTA tile is 128 output channels (the UMMA M dimension) x MT tokens
//     (the UMMA N dimension, MT = 16 or 32);
//   * TMA streams, per 512-wide K unit, the packed nibbles (2 x [128 x 128 B]
//     boxes, 128-byte swizzle), the x slice (8 x [MT x 64] bf16 boxes,
//     128-byte swizzle, directly in the UMMA B layout) and the 8 scales and
//     8 biases of every row ([128 x 16 B] boxes) into a 3-4 stage ring;
//   * eight dequant warps unpack nibbles in registers (bf16x2 magic-number
//     trick + one bf16x2 FMA per pair, exact against the fp32 formula) and
//     write the bf16 weight tile straight into TMEM with tcgen05.st, one TMEM
//     lane per output channel, 32 columns per 64-wide quant group;
//   * one thread issues tcgen05.mma with A from TMEM and B (x) from shared
//     memory, accumulating fp32 in TMEM (two accumulator buffers);
//   * four epilogue warps drain the accumulator with tcgen05.ld.
// Work is split "stream-K" style: the (tile, K unit) space is cut into one
// contiguous range per CTA (grid = min(#SMs, #units)), so every SM streams
// the same number of bytes whatever N and K are.  Tiles shared by several
// CTAs are reduced through an fp32 workspace; the last CTA to arrive (one
// atomic counter per tile, no spin-waits) sums the partials in CTA order,
// so results are bit-reproducible, writes bf16 and resets the counter.
#include "common.cuh"
#include "host_common.cuh"

namespace dfl {

namespace qmm {

constexpr int BN = 128;           // output channels per tile (UMMA M)
constexpr int UNIT_K = 512;       // K per pipeline stage (8 quant groups)
constexpr int GS = 64;            // quant group size (one TMEM A slot)
constexpr int NSUB = UNIT_K / GS; // 8 sub-blocks per stage
constexpr int A_COLS = 32;        // TMEM columns per A slot (64 bf16 per lane)
constexpr int NUM_WARPS = 14;
constexpr int NUM_THREADS = NUM_WARPS * 32;
constexpr int WARP_TMA = 0;
constexpr int WARP_MMA = 1;
constexpr int WARP_DQ0 = 2;       // warps 2..9 dequantise
constexpr int WARP_EPI0 = 10;     // warps 10..13 drain the accumulator
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL0 = NSUB * A_COLS;  // 256

template <int MT>
struct Cfg {
  static constexpr int PACK_BYTES = BN * UNIT_K / 2;  // 32 KB
  static constexpr int XBLK_BYTES = MT * 128;         // one [MT x 64] bf16 block
  static constexpr int X_BYTES = MT * UNIT_K * 2;
  static constexpr int SB_BYTES = BN * 16;            // 8 bf16 per row
  static constexpr int STAGE_BYTES = PACK_BYTES + X_BYTES + 2 * SB_BYTES;
  static constexpr int NSTAGE = (MT <= 16) ? 4 : 3;
  static constexpr int OFF_X = PACK_BYTES;
  static constexpr int OFF_S = PACK_BYTES + X_BYTES;
  static constexpr int OFF_B = OFF_S + SB_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = NSTAGE * STAGE_BYTES + BAR_BYTES + 1024;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(XBLK_BYTES % 1024 == 0, "x blocks must keep 1024-byte alignment");
  static_assert(ACC_COL0 + 2 * MT <= TMEM_COLS, "TMEM budget");
};

struct Params {
  const uint16_t* x;       // only used when scales need plain loads
  const uint16_t* scales;  // [N, K/64]
  const uint16_t* biases;  // [N, K/64]
  uint16_t* y;             // [M, N]
  float* partials;         // [grid][2][MT][BN]
  int* counters;           // [n_tiles]
  int M, K, N;
  int n_tiles, k_units, total_units, grid;
  int sb_tma;              // scales/biases via TMA (K % 512 == 0)
};

__device__ __forceinline__ int unit_begin(int c, int total, int grid) {
  return int((long long)c * total / grid);
}

// First CTA whose unit range contains unit u.
__device__ __forceinline__ int cta_of_unit(int u, int total, int grid) {
  // largest c with floor(c * total / grid) <= u
  long long c = ((long long)(u + 1) * grid + total - 1) / total - 1;
  return int(c);
}

// Eight nibbles (one packed word, low nibble first) -> four bf16x2 words in
// natural K order: w = nib * s + b with a single rounding to bf16.
__device__ __forceinline__ void dequant8(uint32_t q, __nv_bfloat162 s2, __nv_bfloat162 b2,
                                         uint32_t* out) {
  const uint32_t kMagic = 0x43004300u;  // bf16x2 (128, 128); low mantissa bits carry n
  const uint32_t a = (q & 0x000F000Fu) | kMagic;          // (n0, n4)
  const uint32_t b = ((q >> 4) & 0x000F000Fu) | kMagic;   // (n1, n5)
  const uint32_t c = ((q >> 8) & 0x000F000Fu) | kMagic;   // (n2, n6)
  const uint32_t d = ((q >> 12) & 0x000F000Fu) | kMagic;  // (n3, n7)
  uint32_t p[4];
  p[0] = __byte_perm(a, b, 0x5410);  // (n0, n1)
  p[1] = __byte_perm(c, d, 0x5410);  // (n2, n3)
  p[2] = __byte_perm(a, b, 0x7632);  // (n4, n5)
  p[3] = __byte_perm(c, d, 0x7632);  // (n6, n7)
  const __nv_bfloat162 k128 = __halves2bfloat162(__ushort_as_bfloat16(0x4300),
                                                 __ushort_as_bfloat16(0x4300));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&p[i]);
    v = __hsub2(v, k128);            // exact: integer n in bf16
    v = __hfma2(v, s2, b2);          // n * s + b, one rounding
    out[i] = *reinterpret_cast<const uint32_t*>(&v);
  }
}

__device__ __forceinline__ __nv_bfloat162 splat_bf16(uint32_t word, int half) {
  const uint16_t h = half ? uint16_t(word >> 16) : uint16_t(word & 0xFFFFu);
  const __nv_bfloat16 v = __ushort_as_bfloat16(h);
  return __halves2bfloat162(v, v);
}

template <int MT>
__device__ __forceinline__ void epilogue_load(uint32_t taddr, float (&acc)[MT]) {
  uint32_t r[16];
#pragma unroll
  for (int c = 0; c < MT; c += 16) {
    tmem_ld_32x32b_x16(taddr + c, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[c + i] = __uint_as_float(r[i]);
  }
}

template <int MT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    qmm_w4g64_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_b,
                     const Params p) {
  using C = Cfg<MT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::NSTAGE * C::STAGE_BYTES);
  uint64_t* full = bars;                       // [NSTAGE]  TMA landed
  uint64_t* empty = full + C::NSTAGE;          // [NSTAGE]  stage consumed
  uint64_t* afull = empty + C::NSTAGE;         // [NSUB]    TMEM A slot written
  uint64_t* aempty = afull + NSUB;             // [NSUB]    TMEM A slot read by MMA
  uint64_t* accfull = aempty + NSUB;           // [2]
  uint64_t* accempty = accfull + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
  int* flag_slot = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int u0 = unit_begin(cta, p.total_units, p.grid);
  const int u1 = unit_begin(cta + 1, p.total_units, p.grid);
  const int n_units = u1 - u0;
  const int ku = p.k_units;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NSTAGE; ++i) {
      mbar_init(&full[i], p.sb_tma ? 1 : 2);
      mbar_init(&empty[i], 8 + 1);
    }
    for (int i = 0; i < NSUB; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == WARP_MMA) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_x);
      if (p.sb_tma) {
        tma_prefetch_desc(&tm_s);
        tma_prefetch_desc(&tm_b);
      }
    }
    const int groups = p.K / GS;
    for (int it = 0; it < n_units; ++it) {
      const int s = it % C::NSTAGE;
      const uint32_t ph = (it / C::NSTAGE) & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&empty[s], ph ^ 1);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      const int u = u0 + it;
      const int tile = u / ku;
      const int kb = u - tile * ku;
      const int n0 = tile * BN;
      const int k0 = kb * UNIT_K;
      uint8_t* st = smem + s * C::STAGE_BYTES;
      if (lane == 0) {
        const uint32_t bytes = C::PACK_BYTES + C::X_BYTES + (p.sb_tma ? 2 * C::SB_BYTES : 0);
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d(st, &tm_w, &full[s], k0 / 8, n0);
        tma_load_2d(st + C::PACK_BYTES / 2, &tm_w, &full[s], k0 / 8 + 32, n0);
#pragma unroll
        for (int b = 0; b < NSUB; ++b)
          tma_load_2d(st + C::OFF_X + b * C::XBLK_BYTES, &tm_x, &full[s], k0 + b * GS, 0);
        if (p.sb_tma) {
          tma_load_2d(st + C::OFF_S, &tm_s, &full[s], k0 / GS, n0);
          tma_load_2d(st + C::OFF_B, &tm_b, &full[s], k0 / GS, n0);
        }
      }
      if (!p.sb_tma) {
        // Row strides of scales/biases are not 16-byte multiples: plain loads.
        uint16_t* ss = reinterpret_cast<uint16_t*>(st + C::OFF_S);
        uint16_t* sbv = reinterpret_cast<uint16_t*>(st + C::OFF_B);
        const int g0 = k0 / GS;
        for (int i = lane; i < BN * 8; i += 32) {
          const int r = i >> 3, gi = i & 7;
          const int n = n0 + r, g = g0 + gi;
          uint16_t sv = 0, bv = 0;
          if (n < p.N && g < groups) {
            sv = p.scales[(size_t)n * groups + g];
            bv = p.biases[(size_t)n * groups + g];
          }
          ss[i] = sv;
          sbv[i] = bv;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
    }
  } else if (warp == WARP_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BN, MT);
      int acc_it = 0;
      uint32_t buf = 0;
      for (int it = 0; it < n_units; ++it) {
        const int s = it % C::NSTAGE;
        const uint32_t ph = (it / C::NSTAGE) & 1;
        const int kb = (u0 + it) % ku;
        const bool seg_start = (it == 0) || (kb == 0);
        const bool seg_end = (it == n_units - 1) || (kb == ku - 1);
        if (seg_start) {
          buf = acc_it & 1;
          if (!mbar_wait(&accempty[buf], ((acc_it >> 1) & 1) ^ 1)) break;
          tc_fence_after();
        }
        if (!mbar_wait(&full[s], ph)) break;
        const uint32_t xbase = smem_u32(smem + s * C::STAGE_BYTES + C::OFF_X);
        const uint32_t d_tmem = tmem_base + ACC_COL0 + buf * MT;
        bool ok = true;
        for (int sb = 0; sb < NSUB; ++sb) {
          if (!mbar_wait(&afull[sb], it & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < GS / 16; ++k4) {
            const uint32_t a_tmem = tmem_base + sb * A_COLS + k4 * 8;
            const uint64_t bdesc = make_sw128_desc(xbase + sb * C::XBLK_BYTES + k4 * 32);
            const uint32_t accum = (seg_start && sb == 0 && k4 == 0) ? 0u : 1u;
            mma_bf16_ts(d_tmem, a_tmem, bdesc, idesc, accum);
          }
          tc_commit(&aempty[sb]);
        }
        if (!ok) break;
        tc_commit(&empty[s]);
        if (seg_end) {
          tc_commit(&accfull[buf]);
          ++acc_it;
        }
      }
    }
    __syncwarp();
  } else if (warp < WARP_EPI0) {
    // ------------------------------------------------------------ dequant
    const int dw = warp - WARP_DQ0;
    const int grp = dw >> 2;              // handles sub-blocks with sb % 2 == grp
    const int quad = warp & 3;            // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;       // output channel within the tile
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    for (int it = 0; it < n_units; ++it) {
      const int s = it % C::NSTAGE;
      const uint32_t ph = (it / C::NSTAGE) & 1;
      if (!mbar_wait(&full[s], ph)) break;
      const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
      const uint4 sv = ld_shared_v4(st + C::OFF_S + r * 16);
      const uint4 bv = ld_shared_v4(st + C::OFF_B + r * 16);
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
      bool ok = true;
#pragma unroll
      for (int j = 0; j < NSUB / 2; ++j) {
        const int sb = 2 * j + grp;
        if (!mbar_wait(&aempty[sb], (it & 1) ^ 1)) { ok = false; break; }
        tc_fence_after();
        const int box = sb >> 2;
        const int c0 = 2 * (sb & 3);
        const uint32_t rowb = st + box * (C::PACK_BYTES / 2) + r * 128;
        const uint4 q0 = ld_shared_v4(rowb + (uint32_t((c0 ^ (r & 7))) << 4));
        const uint4 q1 = ld_shared_v4(rowb + (uint32_t(((c0 + 1) ^ (r & 7))) << 4));
        // group sb = 2j + grp lives in word j, half grp
        const __nv_bfloat162 s2 = splat_bf16(sw[j], grp);
        const __nv_bfloat162 b2 = splat_bf16(bw[j], grp);
        uint32_t w[32];
        dequant8(q0.x, s2, b2, &w[0]);
        dequant8(q0.y, s2, b2, &w[4]);
        dequant8(q0.z, s2, b2, &w[8]);
        dequant8(q0.w, s2, b2, &w[12]);
        dequant8(q1.x, s2, b2, &w[16]);
        dequant8(q1.y, s2, b2, &w[20]);
        dequant8(q1.z, s2, b2, &w[24]);
        dequant8(q1.w, s2, b2, &w[28]);
        tmem_st_32x32b_x32(lane_base + sb * A_COLS, w);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[sb]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int et = threadIdx.x - WARP_EPI0 * 32;  // 0..127
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    if (n_units > 0) {
      const int t_first = u0 / ku;
      const int t_last = (u1 - 1) / ku;
      int acc_it = 0;
      for (int t = t_first; t <= t_last; ++t) {
        const int kb0 = (t == t_first) ? (u0 - t * ku) : 0;
        const int kb1 = (t == t_last) ? (u1 - t * ku) : ku;
        const uint32_t buf = acc_it & 1;
        if (!mbar_wait(&accfull[buf], (acc_it >> 1) & 1)) break;
        tc_fence_after();
        float acc[MT];
        epilogue_load<MT>(lane_base + ACC_COL0 + buf * MT, acc);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[buf]);
        ++acc_it;

        const int n = t * BN + r;
        const bool full_tile = (kb0 == 0) && (kb1 == ku);
        if (full_tile) {
          if (n < p.N) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
              if (m < p.M) p.y[(size_t)m * p.N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[m]));
          }
          continue;
        }
        // Partial tile: publish fp32 partial, last arriver reduces.
        const int slot = (u0 >= t * ku) ? 0 : 1;
        float* mine = p.partials + ((size_t)(cta * 2 + slot) * MT) * BN;
#pragma unroll
        for (int m = 0; m < MT; ++m) mine[m * BN + r] = acc[m];
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          const int c_lo = cta_of_unit(t * ku, p.total_units, p.grid);
          const int c_hi = cta_of_unit(t * ku + ku - 1, p.total_units, p.grid);
          const int expected = c_hi - c_lo + 1;
          const int prev = atomicAdd(&p.counters[t], 1);
          *flag_slot = (prev == expected - 1) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (*flag_slot) {
          __threadfence();
          const int c_lo = cta_of_unit(t * ku, p.total_units, p.grid);
          const int c_hi = cta_of_unit(t * ku + ku - 1, p.total_units, p.grid);
          float sum[MT];
#pragma unroll
          for (int m = 0; m < MT; ++m) sum[m] = 0.f;
          for (int c = c_lo; c <= c_hi; ++c) {
            const int cs = (unit_begin(c, p.total_units, p.grid) >= t * ku) ? 0 : 1;
            const float* src = p.partials + ((size_t)(c * 2 + cs) * MT) * BN;
#pragma unroll
            for (int m = 0; m < MT; ++m) sum[m] += __ldcg(src + m * BN + r);
          }
          if (n < p.N) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
              if (m < p.M) p.y[(size_t)m * p.N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(sum[m]));
          }
          if (et == 0) p.counters[t] = 0;
        }
        named_bar_sync(1, 128);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_MMA) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace qmm

}  // namespace dfl

// ============================================================== host side
namespace dfl {
namespace qmm {

inline int choose_mt(int M) { return M <= 16 ? 16 : 32; }

inline void geometry(int M, int K, int N, int num_sms, int* n_tiles, int* k_units, int* total,
                     int* grid) {
  *n_tiles = (N + BN - 1) / BN;
  *k_units = (K + UNIT_K - 1) / UNIT_K;
  *total = *n_tiles * *k_units;
  *grid = *total < num_sms ? *total : num_sms;
}

inline size_t workspace_bytes_for(int M, int K, int N, int num_sms) {
  int n_tiles, k_units, total, grid;
  geometry(M, K, N, num_sms, &n_tiles, &k_units, &total, &grid);
  const int mt = choose_mt(M);
  const size_t part = size_t(grid) * 2 * mt * BN * sizeof(float);
  const size_t cnt = ((size_t(n_tiles) * sizeof(int)) + 255) & ~size_t(255);
  return part + cnt;
}

template <int MT>
int launch(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales, const uint16_t* biases,
           uint16_t* y, void* ws, int M, int K, int N, int num_sms, int dev,
           cudaStream_t stream) {
  using C = Cfg<MT>;
  static std::atomic<uint64_t> smem_done{0};
  int st = host::ensure_smem(qmm_w4g64_kernel<MT>, C::SMEM_BYTES, dev, smem_done);
  if (st != DFL_OK) return st;

  Params p;
  p.x = x;
  p.scales = scales;
  p.biases = biases;
  p.y = y;
  p.M = M;
  p.K = K;
  p.N = N;
  geometry(M, K, N, num_sms, &p.n_tiles, &p.k_units, &p.total_units, &p.grid);
  p.partials = reinterpret_cast<float*>(ws);
  p.counters = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ws) +
                                      size_t(p.grid) * 2 * MT * BN * sizeof(float));
  p.sb_tma = (K % UNIT_K == 0) && host::aligned(scales, 16) && host::aligned(biases, 16);

  CUtensorMap tm_w, tm_x, tm_s, tm_b;
  st = host::make_tmap_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w_q, uint64_t(K / 8), uint64_t(N),
                          uint64_t(K / 2), 32, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != DFL_OK) return st;
  st = host::make_tmap_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, uint64_t(K), uint64_t(M),
                          uint64_t(K) * 2, GS, MT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != DFL_OK) return st;
  if (p.sb_tma) {
    st = host::make_tmap_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, scales, uint64_t(K / GS),
                            uint64_t(N), uint64_t(K / GS) * 2, 8, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != DFL_OK) return st;
    st = host::make_tmap_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, biases, uint64_t(K / GS),
                            uint64_t(N), uint64_t(K / GS) * 2, 8, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != DFL_OK) return st;
  } else {
    std::memset(&tm_s, 0, sizeof(tm_s));
    std::memset(&tm_b, 0, sizeof(tm_b));
  }
  qmm_w4g64_kernel<MT><<<p.grid, NUM_THREADS, C::SMEM_BYTES, stream>>>(tm_w, tm_x, tm_s, tm_b, p);
  return host::launch_status();
}

}  // namespace qmm
}  // namespace dfl

extern "C" size_t dfl_verify_qmm_workspace_bytes(int M, int K, int N, int* status) {
  int dummy;
  int* st = status ? status : &dummy;
  if (M < 1 || M > 32 || K < 64 || K % 64 != 0 || N < 1) {
    *st = DFL_ERR_BAD_SHAPE;
    return 0;
  }
  int dev, sms;
  *st = dfl::host::current_device(&dev, &sms);
  if (*st != DFL_OK) return 0;
  return dfl::qmm::workspace_bytes_for(M, K, N, sms);
}

extern "C" int dfl_verify_qmm_w4g64(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                                    const uint16_t* biases, uint16_t* y, void* workspace,
                                    size_t workspace_bytes, int M, int K, int N, void* stream) {
  if (M < 1 || M > 32 || K < 64 || K % 64 != 0 || N < 1) return DFL_ERR_BAD_SHAPE;
  if (!x || !w_q || !scales || !biases || !y) return DFL_ERR_NULL_POINTER;
  if (!dfl::host::aligned(x, 16) || !dfl::host::aligned(w_q, 16) ||
      !dfl::host::aligned(scales, 2) || !dfl::host::aligned(biases, 2) ||
      !dfl::host::aligned(y, 2))
    return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = dfl::host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  const size_t need = dfl::qmm::workspace_bytes_for(M, K, N, sms);
  if (!workspace || workspace_bytes < need) return DFL_ERR_WORKSPACE;
  if (!dfl::host::aligned(workspace, 16)) return DFL_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dfl::qmm::choose_mt(M) == 16)
    return dfl::qmm::launch<16>(x, w_q, scales, biases, y, workspace, M, K, N, sms, dev, s);
  return dfl::qmm::launch<32>(x, w_q, scales, biases, y, workspace, M, K, N, sms, dev, s);
}
