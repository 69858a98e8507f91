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
//     (the UMMA N dimension, MT = 16 or 32); one CTA per SM, 25 warps;
//   * the pipeline unit is 512 of K (8 quant groups).  The producer warp
//     streams the packed nibbles by TMA (2 boxes of [128 rows x 128 B],
//     128-byte swizzle) into a 4-stage ring and the scales / biases in
//     4-unit chunks into a 2-slot ring, without waiting for the previous
//     launch (programmatic dependent launch);
//   * 16 dequant warps (4 groups x 4 TMEM lane quadrants, thread = output
//     channel) unpack nibbles in registers: 3 shifts + 4 LOP3 per word give
//     128 + n exactly, then per pair one exact bf16x2 FMA (v - 128) and one
//     bf16x2 FMA n * s + b with a single rounding.  MLX-packed words come out
//     in the within-8 K order 0,4,1,5,2,6,3,7, pair-packed words (PW) in
//     natural order; tiles go to 12 rotating TMEM A slots with tcgen05.st;
//   * x: with PW weights one x-warp thread loads it by TMA straight into a
//     4-slot ring; with MLX packing the x warps stage it and permute each
//     16-byte chunk to the within-8 order; grouped (MoE) mode gathers rows;
//   * four MMA warps each own an accumulator and two of the eight sub-blocks
//     of a unit and only wait and issue (one MMA per ~64+ cycles per thread
//     at N = 16, so four issuers are needed);
//   * the x warps run the epilogue (TMEM -> registers -> y; with SILU the
//     gate/up pairs of a warp's lanes are combined by one shuffle).
// Work is split "stream-K" style: the (tile, K unit) space is cut into one
// contiguous range per CTA (grid = min(#SMs, #units)), ranges computed on the
// host and skewed towards the CTAs that start first.  A tile shared by CTAs
// c_lo..c_hi is the last of c_lo's range: the others store tagged fp32
// partials (low mantissa bit set), c_lo's dequant warps poll, sum them in
// CTA order and clear them, and its epilogue adds its own accumulator, so
// results are bit-reproducible.
#include "common.cuh"
#include "host_common.cuh"

namespace dfl {

namespace qmm {

constexpr int BN = 128;           // output channels per tile (UMMA M)
constexpr int kMaxGrid = 160;     // CTAs of a dense launch (one per SM; B200 has 148)
constexpr int UNIT_K = 512;       // K per pipeline stage (8 quant groups)
constexpr int GS = 64;            // quant group size (one TMEM A slot)
constexpr int NSUB = UNIT_K / GS; // 8 sub-blocks per stage
constexpr int A_COLS = 32;        // TMEM columns per A slot (64 bf16 per lane)
constexpr int NUM_MMA_WARPS = 4;  // concurrent tcgen05.mma issuers, one accumulator each
constexpr int NDG = 4;            // dequant warp groups (4 warps each)
constexpr int WARP_TMA = 0;
constexpr int WARP_MMA0 = 1;                           // warps 1..4 issue MMAs
constexpr int WARP_DQ0 = WARP_MMA0 + NUM_MMA_WARPS;    // dequant warps
constexpr int WARP_EPI0 = WARP_DQ0 + 4 * NDG;          // 4 x-staging + epilogue warps
constexpr int NUM_WARPS = WARP_EPI0 + 4;
constexpr int NUM_THREADS = NUM_WARPS * 32;
constexpr int TMEM_COLS = 512;
constexpr int SUB_PER_MMA = NSUB / NUM_MMA_WARPS;  // sub-blocks per MMA warp per unit
constexpr int BAR_ID_EPI = 1;            // named barrier of the epilogue warps
constexpr int BAR_ID_RED = 2;            // dequant warps hand the split-K sum to the epilogue
constexpr int BAR_ID_DQ = 3;             // the dequant warps among themselves
constexpr int SBC = 4;                   // units per scale/bias chunk (32 groups)
static_assert(NSUB % NUM_MMA_WARPS == 0, "sub-block split");

template <int MT, bool PW = false>
struct Cfg {
  static constexpr int PACK_BYTES = BN * UNIT_K / 2;  // 32 KB
  static constexpr int STAGE_BYTES = PACK_BYTES;
  static constexpr int NSTAGE = 4;
  // scales / biases: chunks of SBC units (64-byte rows), double-buffered
  static constexpr int SBC_ROW = SBC * NSUB * 2;      // 64 bytes
  static constexpr int SBC_HALF = BN * SBC_ROW;       // scales (or biases) of a chunk
  static constexpr int SBC_BYTES = 2 * SBC_HALF;
  static constexpr int OFF_SB = NSTAGE * STAGE_BYTES;
  static constexpr int XBLK_BYTES = MT * 128;         // one [MT x 64] bf16 block
  static constexpr int XSLOT_BYTES = NSUB * XBLK_BYTES;  // one unit of x
  // x ring depth (units); pair-packed weights have no permute step and
  // use the smem it leaves for one more slot at MT = 16
  static constexpr int XS = (MT <= 16) ? (PW ? 4 : 3) : 2;
  static constexpr int OFF_XRING = OFF_SB + 2 * SBC_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_BYTES = OFF_XRING + XS * XSLOT_BYTES + BAR_BYTES + 1024;
  // x chunks (16 bytes = 8 bf16) per unit, and per x-staging thread.
  static constexpr int X_CHUNKS = NSUB * MT * 8;
  static constexpr int X_PER_THREAD = X_CHUNKS / 128;
  static constexpr int NACC = NUM_MMA_WARPS;
  static constexpr int ACC_COLS = NACC * MT;  // one accumulator buffer
  // TMEM A slots (one quant group of the dequantised tile each): 1.5 units
  // when the accumulators leave room, so dequant can run ahead of the MMAs.
  static constexpr int NASLOT = (MT <= 16) ? 12 : 8;
  static constexpr int ACC_COL0 = NASLOT * A_COLS;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(XBLK_BYTES % 1024 == 0, "x blocks must keep 1024-byte alignment");
  static_assert(X_CHUNKS % 128 == 0, "x chunks per thread");
  static_assert(ACC_COL0 + 2 * ACC_COLS <= TMEM_COLS, "TMEM budget");
  static_assert(NASLOT % NDG == 0 && NASLOT % NUM_MMA_WARPS == 0 && NASLOT >= NSUB, "A slots");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

struct Params {
  const uint16_t* x;       // [M, K]
  const uint16_t* scales;  // [N, K/64]
  const uint16_t* biases;  // [N, K/64]
  uint16_t* y;             // [M, N]
  float* partials;         // [grid][MT][BN], low mantissa bit = valid
  int M, K, N;
  int n_tiles, k_units, total_units, grid;
  int sb_tma;              // scales/biases rows are 16-byte multiples (TMA path)
  // Grouped (MoE expert) mode: problem pi multiplies g_m[pi] <= 16 rows of x,
  // gathered through g_rows[pi][*], with expert g_expert[pi]'s weights and
  // scatters them to rows g_out[pi][*] of y.  The problem count lives in
  // device memory (g_count) so routing never needs a host round trip.
  const int* g_count;
  const int* g_expert;
  const int* g_m;
  const int* g_rows;       // [P][16]
  const int* g_out;        // [P][16]
  int tpp;                 // 128-row tiles per problem (all tiles when dense)
  int table_ready;         // grouped: the route table predates the previous launch
  // Dense: first unit of every CTA's stream-K range, ubeg[grid] = total
  // (computed on the host, see split_ranges).  Grouped launches know their
  // unit count only on the device and split evenly.
  int ubeg[kMaxGrid + 1];
};

__device__ __forceinline__ int unit_begin(const Params& p, bool grouped, int c, int total) {
  if (grouped) return int((long long)c * total / p.grid);
  return p.ubeg[c];
}

// The CTA whose (non-empty) unit range contains unit u: the largest c with
// unit_begin(c) <= u.
__device__ __forceinline__ int cta_of_unit(const Params& p, bool grouped, int u, int total) {
  if (grouped) {
    const long long c = ((long long)(u + 1) * p.grid + total - 1) / total - 1;
    return int(c);
  }
  int lo = 0, hi = p.grid - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.ubeg[mid] <= u)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// Eight nibbles (one packed word, low nibble first) -> four bf16x2 words
// w = nib * s + b with a single rounding to bf16.  The pairs come out in the
// K order (0,4), (1,5), (2,6), (3,7): each is one shift + one LOP3 (mask and
// exponent bits), with no byte permutes.  The x operand gets the same
// within-8 permutation (permute_x_chunk), so the MMA still sums x_k * w_k.
template <bool F16>
__device__ __forceinline__ void dequant8(uint32_t q, uint32_t s, uint32_t b, uint32_t* out) {
  // Written in PTX so that each step is exactly one instruction: 3 shifts
  // and 4 LOP3 (mask | exponent bits of the magic value: bf16 0x4300 = 128.0,
  // fp16 0x6400 = 1024.0) on the integer pipe, then per pair an exact x2 FMA
  // (v * 1 - magic = n) and the scale/bias FMA with a single rounding.
  if constexpr (F16) {
    asm("{\n\t.reg .b32 h1, h2, h3, t0, t1, t2, t3;\n\t"
        "shr.b32 h1, %4, 4;\n\t"
        "shr.b32 h2, %4, 8;\n\t"
        "shr.b32 h3, %4, 12;\n\t"
        "lop3.b32 t0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t1, h1, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t2, h2, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t3, h3, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "fma.rn.f16x2 t0, t0, %7, %8;\n\t"
        "fma.rn.f16x2 t1, t1, %7, %8;\n\t"
        "fma.rn.f16x2 t2, t2, %7, %8;\n\t"
        "fma.rn.f16x2 t3, t3, %7, %8;\n\t"
        "fma.rn.f16x2 %0, t0, %5, %6;\n\t"
        "fma.rn.f16x2 %1, t1, %5, %6;\n\t"
        "fma.rn.f16x2 %2, t2, %5, %6;\n\t"
        "fma.rn.f16x2 %3, t3, %5, %6;\n\t}"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
        : "r"(q), "r"(s), "r"(b), "r"(0x3C003C00u), "r"(0xE400E400u));
  } else {
    asm("{\n\t.reg .b32 h1, h2, h3, t0, t1, t2, t3;\n\t"
        "shr.b32 h1, %4, 4;\n\t"
        "shr.b32 h2, %4, 8;\n\t"
        "shr.b32 h3, %4, 12;\n\t"
        "lop3.b32 t0, %4, 0x000F000F, 0x43004300, 0xEA;\n\t"
        "lop3.b32 t1, h1, 0x000F000F, 0x43004300, 0xEA;\n\t"
        "lop3.b32 t2, h2, 0x000F000F, 0x43004300, 0xEA;\n\t"
        "lop3.b32 t3, h3, 0x000F000F, 0x43004300, 0xEA;\n\t"
        "fma.rn.bf16x2 t0, t0, %7, %8;\n\t"
        "fma.rn.bf16x2 t1, t1, %7, %8;\n\t"
        "fma.rn.bf16x2 t2, t2, %7, %8;\n\t"
        "fma.rn.bf16x2 t3, t3, %7, %8;\n\t"
        "fma.rn.bf16x2 %0, t0, %5, %6;\n\t"
        "fma.rn.bf16x2 %1, t1, %5, %6;\n\t"
        "fma.rn.bf16x2 %2, t2, %5, %6;\n\t"
        "fma.rn.bf16x2 %3, t3, %5, %6;\n\t}"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
        : "r"(q), "r"(s), "r"(b), "r"(0x3F803F80u), "r"(0xC300C300u));
  }
}

// fp32 accumulator -> the activation dtype's bits.
template <bool F16>
__device__ __forceinline__ uint16_t to_out16(float v) {
  if constexpr (F16)
    return __half_as_ushort(__float2half_rn(v));
  else
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}


// Reorders the 8 bf16 of a 16-byte x chunk from k = 0..7 to the order the
// dequantised A operand uses: 0, 4, 1, 5, 2, 6, 3, 7.
__device__ __forceinline__ uint4 permute_x_chunk(uint4 v) {
  uint4 r;
  r.x = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
  r.y = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
  r.z = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
  r.w = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
  return r;
}

// Sum the NACC accumulators of one buffer (accumulator a at columns
// taddr + a * MT) in order a = 0..NACC-1.
template <int MT, int NACC>
__device__ __forceinline__ void epilogue_load(uint32_t taddr, float (&acc)[MT]) {
  uint32_t r[16];
#pragma unroll
  for (int c = 0; c < MT; c += 16) {
#pragma unroll
    for (int a = 0; a < NACC; ++a) {
      tmem_ld_32x32b_x16(taddr + a * MT + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i)
        acc[c + i] = (a == 0) ? __uint_as_float(r[i]) : acc[c + i] + __uint_as_float(r[i]);
    }
  }
}

// Byte offset of 16-byte chunk c of row r in a [rows x 64 B] tile written by
// TMA with the 64-byte swizzle (chunk index XOR bits 7-8 of the address).
__device__ __forceinline__ uint32_t sw64_offset(int r, int c) {
  return uint32_t(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// The x chunks (16 bytes = 8 bf16) x-staging thread et (0..127) handles for
// the unit starting at k0: idx = et + 128 * t = (b * MT + r) * 8 + c is
// chunk c of token row r in K block b.  Rows >= M and columns >= K read 0.
template <int MT, bool GROUPED>
__device__ __forceinline__ void load_x_unit(const Params& p, int k0, int pi, int et,
                                            uint4 (&xr)[Cfg<MT>::X_PER_THREAD]) {
  const int rows = GROUPED ? p.g_m[pi] : p.M;
#pragma unroll
  for (int t = 0; t < Cfg<MT>::X_PER_THREAD; ++t) {
    const int idx = et + 128 * t;
    const int c = idx & 7;
    const int r = (idx >> 3) % MT;
    const int b = idx / (MT * 8);
    const int k = k0 + b * GS + c * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows && k < p.K) {
      const int xrow = GROUPED ? p.g_rows[pi * 16 + r] : r;
      v = __ldg(reinterpret_cast<const uint4*>(p.x + (size_t)xrow * p.K + k));
    }
    xr[t] = v;
  }
}

// Permute and store them into a ring slot: block b at b * XBLK_BYTES, UMMA
// K-major with 128-byte swizzle (chunk c of row r at r*128 + ((c ^ (r&7)) << 4)).
template <int MT>
__device__ __forceinline__ void store_x_unit(uint32_t slot, int et,
                                             const uint4 (&xr)[Cfg<MT>::X_PER_THREAD]) {
#pragma unroll
  for (int t = 0; t < Cfg<MT>::X_PER_THREAD; ++t) {
    const int idx = et + 128 * t;
    const int c = idx & 7;
    const int r = (idx >> 3) % MT;
    const int b = idx / (MT * 8);
    st_shared_v4(slot + b * Cfg<MT>::XBLK_BYTES + r * 128 + (uint32_t((c ^ (r & 7))) << 4),
                 permute_x_chunk(xr[t]));
  }
}

// Sum, in CTA order, of the split-K partials of CTAs c_first..c_last (the
// contributors of the tile the calling CTA reduces), element tid + 512 j of
// the [MT][BN] tile for j < EPT.  A partial word is valid once its lowest bit
// is set (contributors tag what they store; a consumed slot is cleared to 0
// here for the next call), so each word is polled until valid, bounded like
// every other wait: past kWaitLimitNs it records kDevWaitTimeout and sets
// the CTA abort word.
template <int MT>
__device__ __forceinline__ void reduce_partials(const Params& p, int c_first, int c_last, int tid,
                                                volatile int* abort_word,
                                                float (&sum)[MT * BN / (32 * 4 * NDG)]) {
  constexpr int NT = 32 * 4 * NDG;
  constexpr int EPT = MT * BN / NT;
  constexpr int QB = 16 / EPT;  // sources per batch: 16 words in flight per thread
#pragma unroll
  for (int j = 0; j < EPT; ++j) sum[j] = 0.f;
  uint32_t* base = reinterpret_cast<uint32_t*>(p.partials);
  for (int c0 = c_first; c0 <= c_last; c0 += QB) {
    if (*abort_word) return;
    const int nq = (c_last - c0 + 1) < QB ? (c_last - c0 + 1) : QB;
    uint32_t v[QB][EPT];
#pragma unroll
    for (int q = 0; q < QB; ++q)
#pragma unroll
      for (int j = 0; j < EPT; ++j)
        v[q][j] = q < nq ? ld_relaxed_u32(base + size_t(c0 + q) * MT * BN + tid + NT * j) : 1u;
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
      bool all = true;
#pragma unroll
      for (int q = 0; q < QB; ++q)
#pragma unroll
        for (int j = 0; j < EPT; ++j)
          if (!(v[q][j] & 1u)) {
            all = false;
            v[q][j] = ld_relaxed_u32(base + size_t(c0 + q) * MT * BN + tid + NT * j);
          }
      if (all) break;
      if (*abort_word) return;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicExch(&g_device_error, kDevWaitTimeout);
        *abort_word = 1;
        return;
      }
    }
#pragma unroll
    for (int q = 0; q < QB; ++q)
#pragma unroll
      for (int j = 0; j < EPT; ++j)
        if (q < nq) {
          sum[j] += __uint_as_float(v[q][j]);
          st_relaxed_u32(base + size_t(c0 + q) * MT * BN + tid + NT * j, 0u);
        }
  }
}

template <int MT, bool GROUPED, bool F16 = false, bool PW = false, bool SILU = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    qmm_w4g64_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                     const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ Params p) {
  static_assert(!(PW && GROUPED), "pair-packed weights: dense layers only");
  // SILU: the weights (of every expert, when grouped) are a gate|up pair
  // interleaved in blocks of 32 rows (16 gate rows, then the 16 up rows of
  // the same outputs); the epilogue writes h = silu(gate) * up, [rows, N / 2],
  // instead of the N projections.
  using C = Cfg<MT, PW>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_XRING + C::XS * C::XSLOT_BYTES);
  uint64_t* full = bars;                       // [NSTAGE]  nibbles + scales landed
  uint64_t* empty = full + C::NSTAGE;          // [NSTAGE]  stage read by the dequant warps
  uint64_t* afull = empty + C::NSTAGE;         // [NASLOT]  TMEM A slot written
  uint64_t* aempty = afull + C::NASLOT;        // [NASLOT]  TMEM A slot read by MMA
  uint64_t* xfull = aempty + C::NASLOT;        // [XS]      x slot staged
  uint64_t* xfree = xfull + C::XS;             // [XS]      x slot read by all MMA warps
  uint64_t* xtma = xfree + C::XS;              // [XS]      x slot landed (dense: TMA)
  uint64_t* sbfull = xtma + C::XS;             // [2]       scale/bias chunk landed
  uint64_t* sbempty = sbfull + 2;              // [2]       chunk read by the dequant warps
  uint64_t* accfull = sbempty + 2;             // [2]
  uint64_t* accempty = accfull + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto wait = [abort_word](uint64_t* bar, uint32_t parity) {
    return mbar_wait_abortable(bar, parity, abort_word);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int ku = p.k_units;
  const int tpp = p.tpp;
  // Launched with programmatic serialization: the route table of grouped
  // mode may be written by the kernel just before, so grouped CTAs wait for
  // it first unless the caller states that it was complete before the
  // previous launch started.  Otherwise (and in dense mode) only the warps
  // that read x or the workspace and write y wait; weight loads and dequant
  // start at once.
  if (GROUPED && !p.table_ready) griddep_wait();
  const int total = GROUPED ? (*p.g_count) * tpp * ku : p.total_units;
  const int u0 = unit_begin(p, GROUPED, cta, total);
  const int u1 = unit_begin(p, GROUPED, cta + 1, total);
  const int n_units = u1 - u0;

  if (threadIdx.x == 0) {
    // descriptor fetches overlap the set-up below
    tma_prefetch_desc(&tm_w);
    if (!GROUPED) tma_prefetch_desc(&tm_x);
    if (p.sb_tma) {
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_b);
    }
    *abort_word = 0;
    for (int i = 0; i < C::NSTAGE; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4 * NDG);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sbfull[i], 1);
      mbar_init(&sbempty[i], 4 * NDG);
    }
    for (int i = 0; i < C::NASLOT; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < C::XS; ++i) {
      mbar_init(&xfull[i], 4);
      mbar_init(&xfree[i], NUM_MMA_WARPS);
      mbar_init(&xtma[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], NUM_MMA_WARPS);
      mbar_init(&accempty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == WARP_TMA) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------ producer
    // Packed weights (+ scale/bias chunks) into the stage ring, NSTAGE units
    // ahead of the dequant warps.  Weights do not depend on the previous
    // kernel, so this warp never waits for it.  It waits only on dequant
    // progress (stage and chunk release), never on the MMAs: x, whose slots
    // the MMAs release, is requested by the x warps.  Lane 0 waits and
    // issues; the other lanes only help with scale/bias rows that are not
    // 16-byte multiples (K % 512 != 0).
    int w_tile = u0 / ku, w_kb = u0 - (u0 / ku) * ku;
    int w_pi = w_tile / tpp;
    w_tile -= w_pi * tpp;
    int w_e = (GROUPED && n_units > 0) ? p.g_expert[w_pi] : 0;
    int chunk = -1;
    const int groups = p.K / GS;
    auto issue_w = [&](int it) -> bool {
      const int n0 = w_tile * BN;
      if (it == 0 || w_kb % SBC == 0) {
        ++chunk;
        const int cs = chunk & 1;
        if (lane == 0) wait(&sbempty[cs], ((chunk >> 1) & 1) ^ 1);
        __syncwarp();
        if (*abort_word) return false;
        uint8_t* dst = smem + C::OFF_SB + cs * C::SBC_BYTES;
        const int g0 = (w_kb / SBC) * SBC * NSUB;
        if (p.sb_tma) {
          if (lane == 0) {
            mbar_arrive_expect_tx(&sbfull[cs], C::SBC_BYTES);
            tma_load_3d(dst, &tm_s, &sbfull[cs], g0, n0, w_e);
            tma_load_3d(dst + C::SBC_HALF, &tm_b, &sbfull[cs], g0, n0, w_e);
          }
        } else {
          for (int i = lane; i < BN * SBC * NSUB; i += 32) {
            const int r = i / (SBC * NSUB), gi = i - r * (SBC * NSUB);
            const int n = n0 + r, g = g0 + gi;
            uint16_t sv = 0, bv = 0;
            if (n < p.N && g < groups) {
              const size_t idx = ((size_t)w_e * p.N + n) * groups + g;
              sv = p.scales[idx];
              bv = p.biases[idx];
            }
            const uint32_t off = sw64_offset(r, gi >> 3) + (gi & 7) * 2;
            *reinterpret_cast<uint16_t*>(dst + off) = sv;
            *reinterpret_cast<uint16_t*>(dst + C::SBC_HALF + off) = bv;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&sbfull[cs]);
        }
      }
      const int s = it % C::NSTAGE;
      if (lane == 0) {
        wait(&empty[s], ((it / C::NSTAGE) & 1) ^ 1);
        if (!*abort_word) {
          uint8_t* st = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], C::PACK_BYTES);
          tma_load_3d(st, &tm_w, &full[s], w_kb * (UNIT_K / 8), n0, w_e);
          tma_load_3d(st + C::PACK_BYTES / 2, &tm_w, &full[s], w_kb * (UNIT_K / 8) + 32, n0, w_e);
        }
      }
      __syncwarp();
      if (*abort_word) return false;
      if (++w_kb == ku) {
        w_kb = 0;
        if (++w_tile == tpp) {
          w_tile = 0;
          ++w_pi;
          if (GROUPED && it + 1 < n_units) w_e = p.g_expert[w_pi];
        }
      }
      return true;
    };
    for (int it = 0; it < n_units; ++it)
      if (!issue_w(it)) break;
  } else if (warp < WARP_DQ0) {
    // ------------------------------------------------------------ MMA issuers
    // Warp j issues the MMAs of sub-blocks j, j + 4 into accumulator j.  The
    // whole warp runs the loop (waits, descriptors stay warp-uniform) and one
    // elected lane issues each MMA and commit; the loop body is only waits
    // and MMAs, everything else is precomputed.
    const int j = warp - WARP_MMA0;
    {
      constexpr uint32_t idesc = make_idesc_16(BN, MT, F16);
      const uint64_t ring_desc = make_sw128_desc(smem_u32(smem + C::OFF_XRING));
      constexpr uint64_t kSlotDesc = uint64_t(C::XSLOT_BYTES >> 4);
      constexpr uint64_t kBlkDesc = uint64_t(C::XBLK_BYTES >> 4);
      int acc_it = 0;
      uint32_t buf = 0;
      int kb = u0 % ku;
      for (int it = 0; it < n_units; ++it, kb = (kb + 1 == ku) ? 0 : kb + 1) {
        const bool seg_start = (it == 0) || (kb == 0);
        const bool seg_end = (it == n_units - 1) || (kb == ku - 1);
        const int xs = it % C::XS;
        if (seg_start) {
          buf = acc_it & 1;
          wait(&accempty[buf], ((acc_it >> 1) & 1) ^ 1);
        }
        wait(PW ? &xtma[xs] : &xfull[xs], (it / C::XS) & 1);
        const uint32_t d_tmem = tmem_base + C::ACC_COL0 + buf * C::ACC_COLS + j * MT;
        const uint64_t slot_desc = ring_desc + kSlotDesc * xs;
        uint32_t acc0 = seg_start ? 0u : 1u;
#pragma unroll
        for (int i = 0; i < SUB_PER_MMA; ++i) {
          const int sb = j + i * NUM_MMA_WARPS;
          const int g = it * NSUB + sb;  // sub-block sequence number -> A slot
          const int slot = g % C::NASLOT;
          wait(&afull[slot], (g / C::NASLOT) & 1);
          tc_fence_after();
          if (!*abort_word) {
            const uint32_t a_tmem = tmem_base + slot * A_COLS;
            const uint64_t bdesc = slot_desc + kBlkDesc * sb;
            mma_bf16_ts_warp(d_tmem, a_tmem, bdesc, idesc, acc0);
            mma_bf16_ts_warp(d_tmem, a_tmem + 8, bdesc + 2, idesc, 1u);
            mma_bf16_ts_warp(d_tmem, a_tmem + 16, bdesc + 4, idesc, 1u);
            mma_bf16_ts_warp(d_tmem, a_tmem + 24, bdesc + 6, idesc, 1u);
          }
          acc0 = 1u;
          tc_commit_warp(&aempty[slot]);
        }
        tc_commit_warp(&xfree[xs]);
        if (seg_end) {
          tc_commit_warp(&accfull[buf]);
          ++acc_it;
        }
      }
    }
  } else if (warp < WARP_EPI0) {
    // ------------------------------------------------------------ dequant
    const int dw = warp - WARP_DQ0;
    const int grp = dw >> 2;              // handles sub-blocks with sb % NDG == grp
    const int quad = warp & 3;            // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;       // output channel within the tile
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    const uint32_t half_sel = (grp & 1) ? 0x3232u : 0x1010u;  // bf16 half -> both halves
    int kb = u0 % ku;
    int chunk = -1;
    for (int it = 0; it < n_units; ++it, kb = (kb + 1 == ku) ? 0 : kb + 1) {
      if (it == 0 || kb % SBC == 0) {
        if (chunk >= 0) {  // done with the previous scale/bias chunk
          __syncwarp();
          if (lane == 0) mbar_arrive(&sbempty[chunk & 1]);
        }
        ++chunk;
        wait(&sbfull[chunk & 1], (chunk >> 1) & 1);
      }
      const int s = it % C::NSTAGE;
      const uint32_t ph = (it / C::NSTAGE) & 1;
      wait(&full[s], ph);
      const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
      // This warp's sub-blocks of the unit are grp and grp + 4 (quant groups
      // of the same numbers); their scales/biases are halves (grp & 1) of
      // words grp / 2 and grp / 2 + 2 of the unit's 16-byte scale row.
      const uint32_t sbc = smem_u32(smem + C::OFF_SB + (chunk & 1) * C::SBC_BYTES) +
                           sw64_offset(r, kb % SBC) + (grp >> 1) * 4;
      const uint32_t s_w0 = ld_shared_u32(sbc), s_w1 = ld_shared_u32(sbc + 8);
      const uint32_t b_w0 = ld_shared_u32(sbc + C::SBC_HALF), b_w1 = ld_shared_u32(sbc + C::SBC_HALF + 8);
      // This warp's packed words of the unit go to registers at once, so the
      // stage is released before any dequant work and the producer can
      // refill it while this unit is still being converted.
      constexpr int SPW = NSUB / NDG;  // sub-blocks per dequant warp per unit
      static_assert(NSUB % NDG == 0 && SPW == 2, "two sub-blocks per dequant warp");
      uint4 qv[SPW][2];
#pragma unroll
      for (int jj = 0; jj < SPW; ++jj) {
        const int sb = NDG * jj + grp;
        const int c0 = 2 * (sb & 3);
        const uint32_t rowb = st + (sb >> 2) * (C::PACK_BYTES / 2) + r * 128;
        qv[jj][0] = ld_shared_v4(rowb + (uint32_t((c0 ^ (r & 7))) << 4));
        qv[jj][1] = ld_shared_v4(rowb + (uint32_t(((c0 + 1) ^ (r & 7))) << 4));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      // Both sub-blocks are converted and stored before one wait for the
      // stores, so the second conversion overlaps the first store.
      int slots[SPW];
#pragma unroll
      for (int jj = 0; jj < SPW; ++jj) {
        const int sb = NDG * jj + grp;
        const int g = it * NSUB + sb;  // sub-block sequence number -> A slot
        const int slot = g % C::NASLOT;
        slots[jj] = slot;
        wait(&aempty[slot], ((g / C::NASLOT) & 1) ^ 1);
        tc_fence_after();
        const uint4 q0 = qv[jj][0];
        const uint4 q1 = qv[jj][1];
        const uint32_t s2 = __byte_perm(jj ? s_w1 : s_w0, 0, half_sel);
        const uint32_t b2 = __byte_perm(jj ? b_w1 : b_w0, 0, half_sel);
        uint32_t w[32];
        dequant8<F16>(q0.x, s2, b2, &w[0]);
        dequant8<F16>(q0.y, s2, b2, &w[4]);
        dequant8<F16>(q0.z, s2, b2, &w[8]);
        dequant8<F16>(q0.w, s2, b2, &w[12]);
        dequant8<F16>(q1.x, s2, b2, &w[16]);
        dequant8<F16>(q1.y, s2, b2, &w[20]);
        dequant8<F16>(q1.z, s2, b2, &w[24]);
        dequant8<F16>(q1.w, s2, b2, &w[28]);
        tmem_st_32x32b_x32(lane_base + slot * A_COLS, w);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
#pragma unroll
        for (int jj = 0; jj < SPW; ++jj) mbar_arrive(&afull[slots[jj]]);
      }
    }
    // The split-K sum of the tile this CTA reduces (the last of its range):
    // the other CTAs' partials, polled and summed here while this CTA's last
    // MMAs drain, handed to the epilogue through shared memory.
    if (n_units > 0) {
      const int t = (u1 - 1) / ku;
      const int kb0 = (t == u0 / ku) ? (u0 - t * ku) : 0;
      const int kb1 = u1 - t * ku;
      if (!(kb0 == 0 && kb1 == ku) && cta_of_unit(p, GROUPED, t * ku, total) == cta) {
        const int c_hi = cta_of_unit(p, GROUPED, t * ku + ku - 1, total);
        constexpr int NT = 32 * 4 * NDG;
        constexpr int EPT = MT * BN / NT;  // partial-sum elements per dequant thread
        float sum[EPT];
        // The partial slots are shared with the previous launch on the stream
        // (same workspace), which may still be reducing its own: read them
        // only once it has completed.
        griddep_wait();
        reduce_partials<MT>(p, cta + 1, c_hi, threadIdx.x - WARP_DQ0 * 32, abort_word, sum);
        named_bar_sync(BAR_ID_DQ, NT);  // every dequant warp is done with the stage ring
        float* red = reinterpret_cast<float*>(smem);
#pragma unroll
        for (int j = 0; j < EPT; ++j) red[threadIdx.x - WARP_DQ0 * 32 + NT * j] = sum[j];
        named_bar_arrive(BAR_ID_RED, 128 + NT);
      }
    }
  } else {
    // ------------------------------------------------- x staging + epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int et = threadIdx.x - WARP_EPI0 * 32;  // 0..127
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    const uint32_t ring = smem_u32(smem + C::OFF_XRING);
    uint4 xr[GROUPED ? C::X_PER_THREAD : 1];
    // x for unit `ix` goes into slot ix % XS once the MMAs of unit ix - XS
    // have read that slot, XD = XS - 1 units ahead of its permutation, in
    // the UMMA K-major 128-byte-swizzled layout (rows >= M and columns >= K
    // zero).  Dense x arrives in natural K order and each 16-byte chunk is
    // permuted in place (the K permutation stays inside a chunk):
    //   * M <= 16 (X_CP): every thread copies its own chunks with cp.async,
    //     one commit group per unit; these go through L1/L2 and do not queue
    //     behind the weight boxes the producer keeps in the TMA unit;
    //   * M <= 32: one thread requests NSUB TMA boxes of [64 K x MT rows]
    //     (twice the bytes; per-thread copies would cost more issue slots).
    // Grouped: rows are gathered through the route table with plain loads,
    // one unit ahead.
    // Pair-packed weights (PW) dequantise to natural K order: x then goes by
    // TMA straight into its slot, XS units ahead, and the MMAs wait on the
    // copy itself (no permutation, no xfull hand-off).
    constexpr int XD = C::XS - 1;
    constexpr bool X_CP = (MT <= 16) && !PW;
    auto x_chunk = [&](int t, int& b, int& rr, int& c) {
      const int idx = et + 128 * t;
      c = idx & 7;
      rr = (idx >> 3) % MT;
      b = idx / (MT * 8);
    };
    auto issue_x = [&](int ix) {  // X_CP: all x threads; else one thread
      const int xs = ix % C::XS;
      if (ix >= C::XS) wait(&xfree[xs], ((ix / C::XS) - 1) & 1);
      const int k0 = ((u0 + ix) % ku) * UNIT_K;
      if constexpr (X_CP) {
        const uint32_t slot = ring + xs * C::XSLOT_BYTES;
#pragma unroll
        for (int t = 0; t < C::X_PER_THREAD; ++t) {
          int b, rr, c;
          x_chunk(t, b, rr, c);
          const int k = k0 + b * GS + c * 8;
          const bool in = rr < p.M && k < p.K;
          cp_async_16(slot + b * C::XBLK_BYTES + rr * 128 + (uint32_t((c ^ (rr & 7))) << 4),
                      in ? p.x + (size_t)rr * p.K + k : p.x, in ? 16u : 0u);
        }
        cp_async_commit();
      } else {
        if (!*abort_word) {
          uint8_t* dst = smem + C::OFF_XRING + xs * C::XSLOT_BYTES;
          mbar_arrive_expect_tx(&xtma[xs], C::XSLOT_BYTES);
#pragma unroll
          for (int b = 0; b < NSUB; ++b)
            tma_load_2d(dst + b * C::XBLK_BYTES, &tm_x, &xtma[xs], k0 + b * GS, 0);
        }
      }
    };
    auto stage_x = [&](int ix) {
      if constexpr (PW) {
        if (et == 0) issue_x(ix);
        __syncwarp();
        return;
      }
      const int xs = ix % C::XS;
      if constexpr (GROUPED) {
        if (ix >= C::XS) wait(&xfree[xs], ((ix / C::XS) - 1) & 1);
        store_x_unit<MT>(ring + xs * C::XSLOT_BYTES, et, xr);
        if (ix + 1 < n_units) {
          const int un = u0 + ix + 1;
          load_x_unit<MT, GROUPED>(p, (un % ku) * UNIT_K, un / (ku * tpp), et, xr);
        }
      } else {
        const uint32_t slot = ring + xs * C::XSLOT_BYTES;
        if constexpr (X_CP) {
          // groups committed so far: units 0 .. min(ix + XD, n) - 1
          if (ix + XD <= n_units)
            cp_async_wait_group<XD - 1>();
          else
            cp_async_wait_all();
#pragma unroll
          for (int t = 0; t < C::X_PER_THREAD; ++t) {
            int b, rr, c;
            x_chunk(t, b, rr, c);
            const uint32_t a = slot + b * C::XBLK_BYTES + rr * 128 + (uint32_t((c ^ (rr & 7))) << 4);
            st_shared_v4(a, permute_x_chunk(ld_shared_v4(a)));
          }
        } else {
          wait(&xtma[xs], (ix / C::XS) & 1);
#pragma unroll
          for (int t = 0; t < C::X_PER_THREAD; ++t) {
            const uint32_t a = slot + uint32_t(et + 128 * t) * 16u;
            st_shared_v4(a, permute_x_chunk(ld_shared_v4(a)));
          }
        }
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&xfull[xs]);
      if constexpr (!GROUPED) {
        if (ix + XD < n_units) {
          if (X_CP || et == 0) issue_x(ix + XD);
        }
        __syncwarp();
      }
    };
    int staged = 0;  // units of x staged so far
    griddep_wait();
    if (n_units > 0) {
      if constexpr (PW) {
        // stage_x only issues: nothing to prefetch ahead of it
      } else if constexpr (GROUPED) {
        load_x_unit<MT, GROUPED>(p, (u0 % ku) * UNIT_K, u0 / (ku * tpp), et, xr);
      } else {
        if (X_CP || et == 0)
          for (int ix = 0; ix < XD && ix < n_units; ++ix) issue_x(ix);
        __syncwarp();
      }
      if constexpr (PW) {
        // Right after the previous launch completes every CTA asks for x at
        // once; asking for one unit first and the rest once it has landed
        // keeps that burst small, so the first MMAs start sooner.
        stage_x(0);
        staged = 1;
        if (n_units > 1 && et == 0) wait(&xtma[0], 0);
        __syncwarp();
      }
      for (; staged < n_units && staged < C::XS; ++staged) stage_x(staged);
      const int t_first = u0 / ku;
      const int t_last = (u1 - 1) / ku;
      int acc_it = 0;
      for (int t = t_first; t <= t_last; ++t) {
        const int kb0 = (t == t_first) ? (u0 - t * ku) : 0;
        const int kb1 = (t == t_last) ? (u1 - t * ku) : ku;
        // Stage x through this segment's last unit (its MMAs need it) and up
        // to XS - 1 units beyond: staging unit ix waits for the MMAs of unit
        // ix - XS, which is then still inside this segment, so those waits
        // never depend on this segment's epilogue.
        const int seg_last = t * ku + kb1 - 1 - u0;
        for (; staged < n_units && staged <= seg_last + C::XS - 1; ++staged) stage_x(staged);
        const uint32_t buf = acc_it & 1;
        // all four epilogue warps agree before leaving (they share BAR_ID_EPI)
        if (!named_bar_and(BAR_ID_EPI, 128, wait(&accfull[buf], (acc_it >> 1) & 1))) break;
        tc_fence_after();
        float acc[MT];
        epilogue_load<MT, C::NACC>(lane_base + C::ACC_COL0 + buf * C::ACC_COLS, acc);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[buf]);
        ++acc_it;

        const int pi = t / tpp;
        const int n = (t - pi * tpp) * BN + r;
        const int rows = GROUPED ? p.g_m[pi] : p.M;
        const int* outrow = GROUPED ? p.g_out + pi * 16 : nullptr;
        // Final values of this thread's output channel n -> y.  With SILU,
        // lanes 0-15 of each warp hold gate channels and lanes 16-31 the up
        // channels of the same h columns (N % 32 == 0, so validity is
        // warp-uniform); both are rounded to the activation dtype first, as
        // the separate projections would be.
        auto store_final = [&](const float (&v)[MT]) {
          if (n >= p.N) return;
          if constexpr (SILU) {
            const int ldh = p.N >> 1;
            const int hcol = (n >> 5) * 16 + (lane & 15);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              const uint32_t mine = to_out16<F16>(v[m]);
              const uint32_t up = __shfl_down_sync(0xffffffffu, mine, 16);
              if (lane < 16 && m < rows)
                p.y[(size_t)(GROUPED ? outrow[m] : m) * ldh + hcol] =
                    silu_mul_bits<F16>(uint16_t(mine), uint16_t(up));
            }
          } else if constexpr (GROUPED) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
              if (m < rows) p.y[(size_t)outrow[m] * p.N + n] = to_out16<F16>(v[m]);
          } else {
            uint16_t* yp = p.y + n;  // walking pointer: no per-row 64-bit index math
#pragma unroll
            for (int m = 0; m < MT; ++m, yp += p.N)
              if (m < rows) *yp = to_out16<F16>(v[m]);
          }
        };
        const bool full_tile = (kb0 == 0) && (kb1 == ku);
        if (full_tile) {
          store_final(acc);
          continue;
        }
        // Partial tile, split over CTAs c_lo..c_hi.  The tile is the last one
        // of c_lo's range and the first (or only) one of every other
        // contributor's.  Contributors store their fp32 partial with the
        // lowest mantissa bit set as a validity tag (a cleared slot reads 0,
        // so no flag or fence round trip is needed); c_lo's dequant warps,
        // idle once its range is converted, poll and sum the other CTAs'
        // partials in CTA order while its own MMAs drain (reduce_partials),
        // and clear the slots for the next call.  The epilogue adds its own
        // accumulator to that sum, so the result is bit-reproducible.
        const int c_lo = cta_of_unit(p, GROUPED, t * ku, total);
        if (cta != c_lo) {
          uint32_t* mine = reinterpret_cast<uint32_t*>(p.partials) + size_t(cta) * MT * BN;
#pragma unroll
          for (int m = 0; m < MT; ++m) st_relaxed_u32(mine + m * BN + r, __float_as_uint(acc[m]) | 1u);
          continue;
        }
        named_bar_sync(BAR_ID_RED, 128 + 32 * 4 * NDG);
        if (*abort_word) break;
        const float* red = reinterpret_cast<const float*>(smem);
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] += red[m * BN + r];
        store_final(acc);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_TMA) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace qmm

}  // namespace dfl

// ============================================================== host side
namespace dfl {
namespace qmm {

inline int choose_mt(int M) { return M <= 16 ? 16 : 32; }

// Reserved area at the start of every workspace; it also bounds the tile
// count of one launch: N <= kMaxTiles * 128.
constexpr size_t kCounterBytes = host::kWorkspaceCounterBytes;
constexpr int kMaxTiles = int(kCounterBytes / sizeof(int));
// Stream-K split skew of the dense launches (see split_ranges).
constexpr int kSplitSkew = 64;

// Largest skew <= want (in steps of 8) that still leaves the last CTA a
// share of at least two units, so that every CTA's range is non-empty (the
// split-K reduction counts one contribution per CTA between the tile's first
// and last CTA).  The mean weight is 1 - skew / 1024 and the last CTA's
// 1 - skew / 256.
inline int clamp_skew(int want, int total, int grid) {
  const double avg = double(total) / grid;
  int skew = want;
  while (skew > 0 && avg * (1.0 - skew / 256.0) / (1.0 - skew / 1024.0) < 2.0) skew -= 8;
  return skew > 0 ? skew : 0;
}

// Stream-K ranges: CTA c takes units [ubeg[c], ubeg[c + 1]).  The first half
// of the CTAs weigh 1 each; from there the weight falls linearly to
// 1 - skew / 256 at the last CTA.  Under programmatic dependent launch the
// CTAs with the highest indices start last (they go to the SMs the previous
// kernel frees last) and their first weights land after the others', so they
// may take fewer units.  skew = 0 is the even split floor(c * total / grid).
inline void split_ranges(int total, int grid, int skew, int* ubeg) {
  const long long h = grid / 2, L = grid - h;
  auto weight = [&](long long c) {
    const long long d = c > h ? c - h : 0;
    return 512LL * L * c - (long long)skew * d * (d + 1);
  };
  const long long wsum = weight(grid);
  for (int c = 0; c <= grid; ++c) ubeg[c] = int((long long)total * weight(c) / wsum);
}

inline void geometry(int M, int K, int N, int num_sms, int* n_tiles, int* k_units, int* total,
                     int* grid) {
  (void)M;
  *n_tiles = (N + BN - 1) / BN;
  *k_units = (K + UNIT_K - 1) / UNIT_K;
  *total = *n_tiles * *k_units;
  const int cap = num_sms < kMaxGrid ? num_sms : kMaxGrid;
  *grid = *total < cap ? *total : cap;
}

inline size_t workspace_bytes_for(int M, int K, int N, int num_sms) {
  int n_tiles, k_units, total, grid;
  geometry(M, K, N, num_sms, &n_tiles, &k_units, &total, &grid);
  const int mt = choose_mt(M);
  return kCounterBytes + size_t(grid) * mt * BN * sizeof(float);
}

// Weight / scale / bias tensor maps over [E, N, K/8] and [E, N, K/64]
// (E = 1 for a dense layer).  Scales and biases go through TMA only when their
// rows are 16-byte multiples (K % 512 == 0).
inline int make_weight_maps(const uint32_t* w_q, const uint16_t* scales, const uint16_t* biases,
                            int E, int K, int N, bool sb_tma, CUtensorMap* tm_w, CUtensorMap* tm_s,
                            CUtensorMap* tm_b) {
  int st = host::make_tmap_3d(tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w_q, uint64_t(K / 8),
                              uint64_t(N), uint64_t(E), uint64_t(K / 2), uint64_t(N) * (K / 2), 32,
                              BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != DFL_OK) return st;
  if (sb_tma) {
    const uint64_t row = uint64_t(K / GS) * 2;
    st = host::make_tmap_3d(tm_s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, scales, uint64_t(K / GS),
                            uint64_t(N), uint64_t(E), row, row * N, SBC * NSUB, BN,
                            CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != DFL_OK) return st;
    st = host::make_tmap_3d(tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, biases, uint64_t(K / GS),
                            uint64_t(N), uint64_t(E), row, row * N, SBC * NSUB, BN,
                            CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != DFL_OK) return st;
  } else {
    std::memset(tm_s, 0, sizeof(*tm_s));
    std::memset(tm_b, 0, sizeof(*tm_b));
  }
  return DFL_OK;
}

template <int MT, bool GROUPED, bool F16 = false, bool PW = false, bool SILU = false>
int launch_kernel(const CUtensorMap& tm_w, const CUtensorMap& tm_s, const CUtensorMap& tm_b,
                  const CUtensorMap& tm_x,
                  const Params& p, int dev, cudaStream_t stream) {
  using C = Cfg<MT, PW>;
  static std::atomic<uint64_t> smem_done{0};
  int st = host::ensure_smem(qmm_w4g64_kernel<MT, GROUPED, F16, PW, SILU>, C::SMEM_BYTES, dev,
                             smem_done);
  if (st != DFL_OK) return st;
  return host::launch_pdl(qmm_w4g64_kernel<MT, GROUPED, F16, PW, SILU>, p.grid,
                          NUM_THREADS, C::SMEM_BYTES, stream,
                          tm_w, tm_s, tm_b, tm_x, p);
}

template <int MT, bool F16 = false, bool PW = false, bool SILU = false>
int launch(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales, const uint16_t* biases,
           uint16_t* y, void* ws, int M, int K, int N, int num_sms, int dev,
           cudaStream_t stream) {
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.x = x;
  p.scales = scales;
  p.biases = biases;
  p.y = y;
  p.M = M;
  p.K = K;
  p.N = N;
  geometry(M, K, N, num_sms, &p.n_tiles, &p.k_units, &p.total_units, &p.grid);
  p.tpp = p.n_tiles;
  split_ranges(p.total_units, p.grid, clamp_skew(kSplitSkew, p.total_units, p.grid), p.ubeg);
  // Workspace layout: [64 KB header, unused by this kernel][one tagged fp32
  // partial slot of MT x BN per CTA]; every kernel leaves the slots zero.
  p.partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kCounterBytes);
  // TMA of scale/bias rows needs 16-byte multiples: K % 512 == 0.
  p.sb_tma = (K % UNIT_K == 0) && host::aligned(scales, 16) && host::aligned(biases, 16);
  CUtensorMap tm_w, tm_s, tm_b, tm_x;
  int st = make_weight_maps(w_q, scales, biases, 1, K, N, p.sb_tma != 0, &tm_w, &tm_s, &tm_b);
  if (st != DFL_OK) return st;
  // x [M, K] bf16 in boxes of [64 K x MT rows], 128-byte swizzle (the UMMA
  // K-major layout); rows >= M read as zero.
  st = host::make_tmap_2d(&tm_x, F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          x, uint64_t(K), uint64_t(M),
                          uint64_t(K) * 2, GS, MT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != DFL_OK) return st;
  return launch_kernel<MT, false, F16, PW, SILU>(tm_w, tm_s, tm_b, tm_x, p, dev, stream);
}

}  // namespace qmm
}  // namespace dfl

extern "C" int dfl_qmm_stream_k_ranges(int total, int grid, int* ubeg, int* skew_used) {
  if (total < 1 || grid < 1 || grid > total || grid > dfl::qmm::kMaxGrid) return DFL_ERR_BAD_SHAPE;
  if (!ubeg) return DFL_ERR_NULL_POINTER;
  const int skew = dfl::qmm::clamp_skew(dfl::qmm::kSplitSkew, total, grid);
  dfl::qmm::split_ranges(total, grid, skew, ubeg);
  if (skew_used) *skew_used = skew;
  return DFL_OK;
}

extern "C" size_t dfl_verify_qmm_workspace_bytes(int M, int K, int N, int* status) {
  int dummy;
  int* st = status ? status : &dummy;
  if (M < 1 || M > 32 || K < 64 || K % 64 != 0 || N < 1 ||
      N > dfl::qmm::kMaxTiles * dfl::qmm::BN) {
    *st = DFL_ERR_BAD_SHAPE;
    return 0;
  }
  int dev, sms;
  *st = dfl::host::current_device(&dev, &sms);
  if (*st != DFL_OK) return 0;
  return dfl::qmm::workspace_bytes_for(M, K, N, sms);
}

namespace dfl {
namespace qmm {
template <bool F16, bool PW = false, bool SILU = false>
int verify_entry(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                 const uint16_t* biases, uint16_t* y, void* workspace, size_t workspace_bytes,
                 int M, int K, int N, void* stream) {
  if (M < 1 || M > 32 || K < 64 || K % 64 != 0 || N < 1 || N > kMaxTiles * BN)
    return DFL_ERR_BAD_SHAPE;
  if (SILU && N % 32 != 0) return DFL_ERR_BAD_SHAPE;
  if (!x || !w_q || !scales || !biases || !y) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(x, 16) || !host::aligned(w_q, 16) || !host::aligned(scales, 2) ||
      !host::aligned(biases, 2) || !host::aligned(y, 2))
    return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  const size_t need = workspace_bytes_for(M, K, N, sms);
  if (!workspace || workspace_bytes < need) return DFL_ERR_WORKSPACE;
  if (!host::aligned(workspace, 16)) return DFL_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (choose_mt(M) == 16)
    return launch<16, F16, PW, SILU>(x, w_q, scales, biases, y, workspace, M, K, N, sms, dev, s);
  return launch<32, F16, PW, SILU>(x, w_q, scales, biases, y, workspace, M, K, N, sms, dev, s);
}

// Pair-packed nibble order: word p of a row holds columns 8p..8p+7 with
// nibble j (bits 4j..4j+3) = column 8p + 2j and nibble 4 + j = column
// 8p + 2j + 1 (j = 0..3).  The dequantiser's shift/mask sequence then yields
// bf16 pairs in natural K order.  Each word maps to itself, so the repack
// may run in place.
__device__ __forceinline__ uint32_t pair_pack_word(uint32_t q) {
  uint32_t r = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    r |= ((q >> (8 * j)) & 0xFu) << (4 * j);             // column 2j     -> nibble j
    r |= ((q >> (8 * j + 4)) & 0xFu) << (4 * (j + 4));   // column 2j + 1 -> nibble 4 + j
  }
  return r;
}

__global__ void repack_pairs_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                    size_t n_vec) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n_vec;
       i += size_t(gridDim.x) * blockDim.x) {
    uint4 v = src[i];
    v.x = pair_pack_word(v.x);
    v.y = pair_pack_word(v.y);
    v.z = pair_pack_word(v.z);
    v.w = pair_pack_word(v.w);
    dst[i] = v;
  }
}
}  // namespace qmm
}  // namespace dfl

extern "C" int dfl_repack_w4_pairs(const uint32_t* src, uint32_t* dst, size_t n_words,
                                   void* stream) {
  if (n_words == 0) return DFL_OK;
  if (!src || !dst) return DFL_ERR_NULL_POINTER;
  if (n_words % 4 != 0) return DFL_ERR_BAD_SHAPE;
  if (!dfl::host::aligned(src, 16) || !dfl::host::aligned(dst, 16)) return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = dfl::host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  const size_t n_vec = n_words / 4;
  const size_t want = (n_vec + 255) / 256;
  const int blocks = int(want < size_t(sms) * 8 ? (want ? want : 1) : size_t(sms) * 8);
  dfl::qmm::repack_pairs_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst), n_vec);
  return dfl::host::launch_status();
}

extern "C" int dfl_verify_qmm_w4g64_pairs(const uint16_t* x, const uint32_t* w_q,
                                          const uint16_t* scales, const uint16_t* biases,
                                          uint16_t* y, void* workspace, size_t workspace_bytes,
                                          int M, int K, int N, void* stream) {
  return dfl::qmm::verify_entry<false, true>(x, w_q, scales, biases, y, workspace,
                                             workspace_bytes, M, K, N, stream);
}

extern "C" int dfl_verify_qmm_w4g64_silu(const uint16_t* x, const uint32_t* w_q,
                                         const uint16_t* scales, const uint16_t* biases,
                                         uint16_t* h, void* workspace, size_t workspace_bytes,
                                         int M, int K, int N, void* stream) {
  return dfl::qmm::verify_entry<false, false, true>(x, w_q, scales, biases, h, workspace,
                                                    workspace_bytes, M, K, N, stream);
}

extern "C" int dfl_verify_qmm_w4g64_pairs_silu(const uint16_t* x, const uint32_t* w_q,
                                               const uint16_t* scales, const uint16_t* biases,
                                               uint16_t* h, void* workspace,
                                               size_t workspace_bytes, int M, int K, int N,
                                               void* stream) {
  return dfl::qmm::verify_entry<false, true, true>(x, w_q, scales, biases, h, workspace,
                                                   workspace_bytes, M, K, N, stream);
}

extern "C" int dfl_verify_qmm_w4g64_pairs_silu_f16(const uint16_t* x, const uint32_t* w_q,
                                                   const uint16_t* scales,
                                                   const uint16_t* biases, uint16_t* h,
                                                   void* workspace, size_t workspace_bytes,
                                                   int M, int K, int N, void* stream) {
  return dfl::qmm::verify_entry<true, true, true>(x, w_q, scales, biases, h, workspace,
                                                  workspace_bytes, M, K, N, stream);
}

extern "C" int dfl_verify_qmm_w4g64_pairs_f16(const uint16_t* x, const uint32_t* w_q,
                                              const uint16_t* scales, const uint16_t* biases,
                                              uint16_t* y, void* workspace,
                                              size_t workspace_bytes, int M, int K, int N,
                                              void* stream) {
  return dfl::qmm::verify_entry<true, true>(x, w_q, scales, biases, y, workspace,
                                            workspace_bytes, M, K, N, stream);
}

extern "C" int dfl_verify_qmm_w4g64(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                                    const uint16_t* biases, uint16_t* y, void* workspace,
                                    size_t workspace_bytes, int M, int K, int N, void* stream) {
  return dfl::qmm::verify_entry<false>(x, w_q, scales, biases, y, workspace, workspace_bytes, M, K,
                                       N, stream);
}

extern "C" int dfl_verify_qmm_w4g64_f16(const uint16_t* x, const uint32_t* w_q,
                                        const uint16_t* scales, const uint16_t* biases,
                                        uint16_t* y, void* workspace, size_t workspace_bytes,
                                        int M, int K, int N, void* stream) {
  return dfl::qmm::verify_entry<true>(x, w_q, scales, biases, y, workspace, workspace_bytes, M, K,
                                      N, stream);
}

// ------------------------------------------------------------------ MoE
namespace dfl {
namespace qmm {

inline void grouped_geometry(int max_problems, int K, int N, int num_sms, int* tpp, int* ku,
                             int* grid) {
  *tpp = (N + BN - 1) / BN;
  *ku = (K + UNIT_K - 1) / UNIT_K;
  const long long units = (long long)max_problems * *tpp * *ku;
  *grid = units < num_sms ? int(units) : num_sms;
}

inline size_t grouped_workspace_bytes(int max_problems, int K, int N, int num_sms) {
  int tpp, ku, grid;
  grouped_geometry(max_problems, K, N, num_sms, &tpp, &ku, &grid);
  return kCounterBytes + size_t(grid) * 16 * BN * sizeof(float);
}

}  // namespace qmm
}  // namespace dfl

extern "C" size_t dfl_moe_qmm_workspace_bytes(int max_problems, int K, int N, int* status) {
  int dummy;
  int* st = status ? status : &dummy;
  if (max_problems < 1 || K < 64 || K % 64 != 0 || N < 1 ||
      (long long)max_problems * ((N + 127) / 128) > dfl::qmm::kMaxTiles) {
    *st = DFL_ERR_BAD_SHAPE;
    return 0;
  }
  int dev, sms;
  *st = dfl::host::current_device(&dev, &sms);
  if (*st != DFL_OK) return 0;
  return dfl::qmm::grouped_workspace_bytes(max_problems, K, N, sms);
}

namespace dfl {
namespace qmm {
template <bool SILU>
int moe_entry(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
              const uint16_t* biases, uint16_t* y, const int32_t* route, int gather_by_pair,
              int max_problems, int E, int K, int N, void* workspace, size_t workspace_bytes,
              void* stream) {
  if (max_problems < 1 || max_problems > E || E < 1 || K < 64 || K % 64 != 0 || N < 1 ||
      (long long)max_problems * ((N + 127) / 128) > kMaxTiles)
    return DFL_ERR_BAD_SHAPE;
  if (SILU && N % 32 != 0) return DFL_ERR_BAD_SHAPE;
  if (!x || !w_q || !scales || !biases || !y || !route) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(x, 16) || !host::aligned(w_q, 16) || !host::aligned(route, 4))
    return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  if (!workspace || workspace_bytes < grouped_workspace_bytes(max_problems, K, N, sms))
    return DFL_ERR_WORKSPACE;
  if (!host::aligned(workspace, 16)) return DFL_ERR_MISALIGNED;
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.x = x;
  p.scales = scales;
  p.biases = biases;
  p.y = y;
  p.M = 16;
  p.K = K;
  p.N = N;
  grouped_geometry(max_problems, K, N, sms, &p.tpp, &p.k_units, &p.grid);
  p.n_tiles = max_problems * p.tpp;
  p.partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kCounterBytes);
  p.sb_tma = (K % UNIT_K == 0) && host::aligned(scales, 16) && host::aligned(biases, 16);
  // route table layout (int32): [0] problem count P, then E expert ids,
  // E row counts, E x 16 token rows, E x 16 pair rows (see dfl_moe_route)
  p.g_count = route;
  p.g_expert = route + 1;
  p.g_m = route + 1 + E;
  p.g_rows = (gather_by_pair & 1) ? route + 1 + 2 * E + 16 * E : route + 1 + 2 * E;
  p.table_ready = (gather_by_pair & 2) ? 1 : 0;
  p.g_out = route + 1 + 2 * E + 16 * E;
  CUtensorMap tm_w, tm_s, tm_b, tm_x;
  std::memset(&tm_x, 0, sizeof(tm_x));  // grouped mode gathers x rows with plain loads
  st = make_weight_maps(w_q, scales, biases, E, K, N, p.sb_tma != 0, &tm_w, &tm_s, &tm_b);
  if (st != DFL_OK) return st;
  return launch_kernel<16, true, false, false, SILU>(tm_w, tm_s, tm_b, tm_x, p, dev,
                                                    reinterpret_cast<cudaStream_t>(stream));
}
}  // namespace qmm
}  // namespace dfl

extern "C" int dfl_moe_qmm_w4g64(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                                 const uint16_t* biases, uint16_t* y, const int32_t* route,
                                 int gather_by_pair, int max_problems, int E, int K, int N,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  return dfl::qmm::moe_entry<false>(x, w_q, scales, biases, y, route, gather_by_pair,
                                    max_problems, E, K, N, workspace, workspace_bytes, stream);
}

extern "C" int dfl_moe_qmm_w4g64_silu(const uint16_t* x, const uint32_t* w_q,
                                      const uint16_t* scales, const uint16_t* biases, uint16_t* h,
                                      const int32_t* route, int gather_by_pair, int max_problems,
                                      int E, int K, int N, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  return dfl::qmm::moe_entry<true>(x, w_q, scales, biases, h, route, gather_by_pair,
                                   max_problems, E, K, N, workspace, workspace_bytes, stream);
}
