// Projection plans: one persistent launch runs a whole sequence of int4 g64
// verify projections (a decoder layer's q|k|v, o, gate|up + SiLU, down, or a
// whole layer stack) at up to 128 token rows per projection: one request's
// 16 verify tokens, or the rows of up to 8 requests sharing one weight read.
//
// Same arithmetic as the per-call qmm (qmm_w4.cu, which replaces the
// reference's M=16 verify kernels, dflash_mlx/verify_qmm.py:196-765, and
// stock mx.quantized_matmul(transpose=True)): w = float(nib) * s + b rounded
// to bf16 (verify_qmm.py:249), fp32 accumulation, bf16 out.  What changes is
// how the work reaches the SMs:
//
//   * Tiled weights (load-time layout, dfl_repack_w4_tiled): every pipeline
//     unit (128 output rows x 512 of K) is one contiguous 36 KB block -- the
//     packed nibbles in the order the dequant threads read them (each warp's
//     16-byte loads are 512 contiguous bytes) followed by the unit's scales
//     and biases (8 bytes per thread).  One bulk copy per unit, streamed with
//     an L2 evict-first hint (weights are read once per step).
//   * Subnormal dequantiser.  A bf16 bit pattern whose exponent field is 0
//     or 1 is worth exactly (bits) * 2^-133, so a nibble masked into bits
//     0-3 of a half word is n * 2^-133 and one in bits 4-7 is n * 2^-129.
//     With the scale stored as s * 2^133 (exact: a power-of-two scaling) one
//     bf16x2 FMA per pair gives n * s + b with a single rounding, the same
//     bits as the reference's dequantisation.  Per 8 weights: 1 shift, 4
//     AND, 4 FMA (the general path needs 3 shifts, 4 LOP3 and 8 FMA).  It
//     needs |s| < 2^-5 for every group; tensors with larger scales use the
//     general "magic 128" path, chosen per projection.
//   * One launch, many projections.  Every CTA walks every projection
//     ("phase") in order and takes an even contiguous share of its
//     (tile, K unit) space (split-K across CTAs as in qmm_w4.cu).  The
//     producer streams the next phase's weights and the dequant warps
//     convert them while the current phase drains, so HBM never waits for a
//     launch boundary.  A phase whose input x is written by an earlier phase
//     names it (dep); its x is loaded only once every CTA has signalled that
//     phase complete (a release counter per phase), so the dataflow of a
//     real forward pass is kept.
//
// Warp roles (one CTA per SM, 26 warps): 0 producer, 1-4 MMA issuers, 5-20
// dequant (4 groups x 4 TMEM lane quadrants, thread = output row), 21-24
// epilogue + split-K reduction + phase signals, 25 x loads.  The token tile
// MT (16, 32, 64 or 128 rows, the UMMA N) is chosen per plan from its
// largest phase.  The four MMA warps issue four independent accumulation
// chains (a chain into one accumulator is latency bound): up to 32 rows as
// four K-interleaved accumulators, at 64 / 128 rows as four token-column
// slices of one accumulator.  Larger tiles stage x in half / quarter units
// and keep fewer weight blocks in flight (the tensor pipe, not HBM, bounds
// them).  A projection over more rows is several phases, one per token tile.
//
// Split-K: a tile shared by CTAs c_lo..c_hi is the last of c_lo's range in
// that phase and the first of the others'.  A contributor stores its fp32
// partial in its own slot (one per CTA and phase parity) and publishes the
// slot with a release store of the phase number; c_lo's epilogue acquires
// that exact stamp, adds the partials to its accumulator in CTA order (so
// results are bit-reproducible) and publishes that it has read them; a
// contributor refills a slot only after its previous partial there was
// read.  Every wait is bounded; a time-out sets the device error word and a
// plan-wide abort word, and every CTA winds down.
#include "common.cuh"
#include "host_common.cuh"

#include <vector>

namespace dfl {
namespace plan {

constexpr int BN = 128;
constexpr int UNIT_K = 512;
constexpr int GS = 64;
constexpr int NSUB = UNIT_K / GS;                      // 8 sub-blocks (quant groups) per unit
constexpr int A_COLS = 32;                             // TMEM columns per A slot
constexpr int NUM_MMA_WARPS = 4;
constexpr int NDG = 4;                                 // dequant warp groups
constexpr int WARP_TMA = 0;
constexpr int WARP_MMA0 = 1;
constexpr int WARP_DQ0 = WARP_MMA0 + NUM_MMA_WARPS;    // 5
constexpr int WARP_EPI0 = WARP_DQ0 + 4 * NDG;          // 21: 4 epilogue warps
constexpr int WARP_X = WARP_EPI0 + 4;                  // 25: x loads
constexpr int NUM_WARPS = WARP_X + 1;                  // 26
constexpr int NUM_THREADS = NUM_WARPS * 32;            // 832
constexpr int TMEM_COLS = 512;
constexpr int BAR_ID_EPI = 1;
constexpr int PACK_BYTES = BN * UNIT_K / 2;            // 32768: nibbles of a unit
constexpr int SB_RECORDS = 4;                          // per row: {s_g, s_g+4, b_g, b_g+4}, g = 0..3
constexpr int SB_BYTES = SB_RECORDS * BN * 8;          // 4096: scales + biases of a unit
constexpr int SPG = NSUB / NDG;                        // sub-blocks per dequant group and unit
constexpr int RPG = SB_RECORDS / NDG;                  // scale/bias records per dequant thread
static_assert(NSUB % NDG == 0 && SB_RECORDS % NDG == 0, "dequant groups");
constexpr int BLK_BYTES = PACK_BYTES + SB_BYTES;       // 36864
constexpr int kMaxGrid = 160;
constexpr int kMaxRows = 128;                         // token rows per phase (one token tile)
constexpr int kMaxPhases = 7936;
constexpr uint32_t kPlanMagic = 0x504C4644u;           // "DFLP"
constexpr int kPlanVersion = 1;
constexpr int kHeaderBytes = 256;
constexpr int kPhaseSilu = 1;                          // DFL_PHASE_SILU
constexpr int kPhaseSubnormal = 2;                     // DFL_PHASE_SUBNORMAL
constexpr int kPhaseGrouped = 4;                       // DFL_PHASE_GROUPED
constexpr int kPhaseScatter = 8;                       // DFL_PHASE_SCATTER
// sorted route table of grouped phases (dfl_moe_sort_pairs): [0] problems P;
// [1 + 2i] first sorted row of problem i (i <= P); [2 + 2i] its expert;
// [kRowMap + r] the pair row (token * top_k + slot) of sorted row r
constexpr int kRouteMaxProblems = 256;
constexpr int kRouteRowMap = 2 + 2 * kRouteMaxProblems;
constexpr int kRouteMaxRows = 256;
constexpr int kMaxGroupedRows = 32;                    // token tile of plans with grouped phases
constexpr int kRouteInts = kRouteRowMap + kRouteMaxRows;
static_assert(kRouteRowMap == 514, "route table layout documented in dflash_b200.h");
// workspace: 64 KB of counter words, then the split-K partial slots
constexpr size_t kCounterBytes = host::kWorkspaceCounterBytes;
constexpr int kWordExit = kMaxPhases;                  // CTAs that finished the launch
constexpr int kWordAbort = kMaxPhases + 1;             // plan-wide abort
constexpr int kWordWhere = kMaxPhases + 2;             // first time-out: (role << 24) | phase
constexpr int kWordWhereCta = kMaxPhases + 3;          // first time-out: CTA
constexpr int kWordDiag = kMaxPhases + 4;              // [8] details of the first time-out
// per CTA and phase parity: the phase (+1) whose partial the slot holds, and
// the phase (+1) whose partial its consumer has read
// split-K partial slots per CTA: one per phase modulo kSlotPhases, so a
// contributor refills a slot only kSlotPhases phases later (its consumer,
// a neighbouring CTA, may lag that far behind before it holds it up)
constexpr int kSlotPhases = 4;
constexpr int kWordReady = kMaxPhases + 16;            // [kMaxGrid][kSlotPhases]
constexpr int kWordConsumed = kWordReady + kSlotPhases * kMaxGrid;  // [kMaxGrid][kSlotPhases]
// per-problem tile counters of grouped phases that a later grouped phase
// reads per problem: [slot][kRouteMaxProblems]
constexpr int kWordProblem = 9472;
constexpr int kMaxProblemSlots = 16;
static_assert(kWordConsumed + kSlotPhases * kMaxGrid <= kWordProblem, "counter region layout");
static_assert((kWordProblem + kMaxProblemSlots * kRouteMaxProblems) * 4 <= int(kCounterBytes),
              "counter region");
// internal phase flag fields (set by the encoder): the problem-counter slot
// (+1) a grouped phase signals per stored tile, and the one it waits on
constexpr int kSignalShift = 8;
constexpr int kWaitShift = 16;
constexpr int kPublicFlags = 0xFF;
// internal phase flag (set by the encoder): y takes 16-byte row stores (y
// 16-byte aligned, ldy and the output width multiples of 8)
constexpr int kVecStore = 1 << 24;
static_assert(BLK_BYTES % 1024 == 0, "stage alignment");

template <int MT>
struct Cfg {
  static_assert(MT == 16 || MT == 32 || MT == 64 || MT == 128, "token tile");
  // MMAs into one accumulator form a dependent chain whose latency, not the
  // tensor pipe, sets the rate, so the four MMA warps issue four independent
  // chains.  Up to 32 tokens each warp takes every fourth sub-block into an
  // accumulator of its own (NACC = 4, summed by the epilogue); at 64 / 128
  // tokens each warp takes one quarter of the token columns (NSLICE = 4,
  // N = 16 / 32 per MMA) of a single accumulator, which keeps the
  // accumulator at MT columns so two buffers fit TMEM beside the A slots.
  static constexpr int NACC = (MT <= 32) ? 4 : 1;
  static constexpr int NSLICE = NUM_MMA_WARPS / NACC;
  static constexpr int SLICE_N = MT / NSLICE;
  static constexpr int NSTAGE = (MT <= 64) ? 4 : 3;    // weight blocks in flight
  static constexpr int XBLK_BYTES = MT * 128;          // one [MT rows x 64 K] bf16 block, SW128
  // x is staged in chunks of XCH sub-blocks (a whole unit up to 32 rows)
  static constexpr int XCH = (MT <= 32) ? NSUB : (MT == 64 ? 4 : 2);
  static constexpr int NCH = NSUB / XCH;               // x chunks per unit
  static constexpr int XCHUNK_BYTES = XCH * XBLK_BYTES;
  static constexpr int XS = (MT <= 16) ? 4 : (MT == 128 ? 3 : 2);   // x ring depth (chunks)
  static constexpr int OFF_XRING = NSTAGE * BLK_BYTES;
  static constexpr int OFF_BARS = OFF_XRING + XS * XCHUNK_BYTES;
  // epilogue staging: per epilogue warp one 16-token pass of its 32 output
  // columns, transposed to token rows (rows padded to 80 bytes)
  static constexpr int STAGE_ROW_BYTES = 80;
  static constexpr int STAGE_WARP_BYTES = 16 * STAGE_ROW_BYTES;
  static constexpr int OFF_STAGE = OFF_BARS + 512;
  static constexpr int SMEM_BYTES = OFF_STAGE + 4 * STAGE_WARP_BYTES + 1024;
  static constexpr int NASLOT = 8;                     // TMEM A slots (one unit)
  static constexpr int ACC_COL0 = NASLOT * A_COLS;
  static constexpr int ACC_COLS = NACC * MT;           // one accumulator buffer
  // accumulator buffers: the MMAs may run this many tile segments ahead of
  // the epilogue (segments are short: 2-10 units per CTA and phase)
  static constexpr int NACCBUF = (MT <= 16) ? 4 : 2;
  // epilogue columns per pass (registers); with
  // one pass the split-K partials are summed before the accumulator is
  // ready, with several they are summed pass by pass
  // x chunks are released by the A-slot release of their last sub-block when
  // every MMA warp reads every sub-block (token slices): that commit already
  // covers all MMAs that read the chunk, and a separate x-release barrier
  // with its own commits costs far more hand-off time per chunk.  Safe when a
  // unit has at least XS chunks: sub-block g + NASLOT (the next use of the
  // A slot) is in a chunk the x loader has not loaded yet when it waits for
  // g, so the slot's barrier is never two phases ahead of that wait.
  static constexpr bool kXReleaseByA = (NSLICE == NUM_MMA_WARPS) && (NCH >= XS);
  static constexpr int EC = 16;
  static constexpr bool kEarlyPartials = (EC == MT);
  // epilogue: at 32+ token rows the accumulator is read in the MMA fragment
  // layout and leaves through stmatrix.trans staging in 16-byte row stores
  // (8x fewer store instructions); 16-row tiles keep one thread per output
  // column and one store per value (fewer live registers in that variant)
  static constexpr bool kFragEpi = (MT >= 32);
  static_assert(ACC_COL0 + NACCBUF * ACC_COLS <= TMEM_COLS, "TMEM budget");
  static constexpr int NUM_BARS = 2 * NSTAGE + 2 * NASLOT + 2 * XS + 2 * NACCBUF + NUM_MMA_WARPS;
  static_assert(NUM_BARS * 8 + 16 <= 512, "barrier area");
  static_assert(XBLK_BYTES % 1024 == 0, "x blocks keep the 1024-byte swizzle alignment");
  static_assert(NASLOT % NDG == 0 && NASLOT >= NSUB, "A slots");
  static_assert(NACC * NSLICE == NUM_MMA_WARPS && XCH % NACC == 0 && NSUB % XCH == 0, "MMA issue split");
  static_assert(SLICE_N % 16 == 0 && (SLICE_N * 128) % 1024 == 0, "token slices: UMMA N, SW128 row groups");
  static_assert(MT % EC == 0 && EC % 16 == 0, "epilogue passes");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// One projection of a plan as the kernel reads it (device memory, 64-byte
// aligned so the x tensor map may be used by TMA in place).
struct alignas(64) Phase {
  CUtensorMap tm_x;      // x [M, K] bf16, box [64 K x MT rows], 128-byte swizzle
  const uint8_t* w;      // tiled blob: n_tiles * ku blocks of BLK_BYTES, tile-major
  uint16_t* y;           // [M, N] (SiLU: [M, N/2]), row stride ldy
  int M, K, N, ldy;
  int n_tiles, ku, total;   // grouped: n_tiles per expert; total from the route table
  int flags, dep;
  int experts;              // grouped phases: experts stacked in w
  const int* route;         // grouped phases: sorted route table
};
static_assert(sizeof(Phase) == 192, "phase record size");

struct Header {
  uint32_t magic;
  int version, n_phases, mt, grid, flags_or;
  // fault injection for tests (dfl_qmm_plan_set_test_fault): a CTA that
  // withholds its split-K partials, and the bound on every wait
  int test_skip_partial_cta;
  int prob_slots;               // problem-counter slots in use
  unsigned long long wait_limit_ns;
  int pad[54];
};
static_assert(sizeof(Header) == kHeaderBytes, "plan header size");

struct RunParams {
  const Phase* phases;
  int n_phases;
  int skip_partial_cta;        // -1 normally
  int prob_slots;
  unsigned long long wait_limit_ns;
  int* words;           // workspace counter words
  float* partials;      // workspace [grid][kSlotPhases][MT][BN]
};

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Untiled bulk copy global -> shared with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_load_hint(uint32_t dst_smem, const void* src, uint32_t bytes,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst_smem),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// 8 pair-packed nibbles (bits 4i..4i+3 = column 2i, bits 16+4i.. = column
// 2i+1) -> 4 bf16x2 words (columns 0-1, 2-3, 4-5, 6-7), subnormal method:
// s_lo = s * 2^133 (fields in bits 0-3 of a half), s_hi = s * 2^129 (bits 4-7).
__device__ __forceinline__ void dequant8_subn(uint32_t q, uint32_t s_lo, uint32_t s_hi, uint32_t b,
                                              uint32_t* out) {
  asm("{\n\t.reg .b32 t, e0, e1, e2, e3;\n\t"
      "shr.b32 t, %4, 8;\n\t"
      "and.b32 e0, %4, 0x000F000F;\n\t"
      "and.b32 e1, %4, 0x00F000F0;\n\t"
      "and.b32 e2, t, 0x000F000F;\n\t"
      "and.b32 e3, t, 0x00F000F0;\n\t"
      "fma.rn.bf16x2 %0, e0, %5, %7;\n\t"
      "fma.rn.bf16x2 %1, e1, %6, %7;\n\t"
      "fma.rn.bf16x2 %2, e2, %5, %7;\n\t"
      "fma.rn.bf16x2 %3, e3, %6, %7;\n\t}"
      : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3])
      : "r"(q), "r"(s_lo), "r"(s_hi), "r"(b));
}

// Same output, general method for any scale: mask | exponent bits of 128.0
// give 128 + n exactly, an exact FMA removes the 128, then n * s + b.
__device__ __forceinline__ void dequant8_magic(uint32_t q, uint32_t s, uint32_t b, uint32_t* out) {
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

// 16 TMEM lanes x 16 columns of 32-bit: thread t gets lanes t/4 and t/4 + 8,
// columns 2(t%4) + {0, 1} and 8 + 2(t%4) + {0, 1} (registers: {lane t/4: c,
// c+1}, {lane t/4+8: c, c+1}, then the same 8 columns further on).
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// Four 8x8 bf16 matrices from the fragment layout (thread t: row t/4, columns
// 2(t%4), 2(t%4)+1 of each) stored transposed; thread 8i + j gives the
// shared address of row j of matrix i.
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                                  uint32_t d) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr),
               "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_relaxed_v4(float* p, float a, float b, float c, float d) {
  asm volatile("st.relaxed.gpu.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ float4 ld_relaxed_v4(const float* p) {
  float4 v;
  asm volatile("ld.relaxed.gpu.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
         (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(0x80008000u));
  return d;
}

// A phase field read through the non-coherent path, issued where it is
// written (volatile) so a role can fetch the next phase's fields one phase
// ahead and never stall on them at a phase boundary.
__device__ __forceinline__ int ld_field(const int* p) {
  int v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ const void* ld_field_ptr(const void* const* p) {
  uint64_t v;
  asm volatile("ld.global.nc.b64 %0, [%1];" : "=l"(v) : "l"(p));
  return reinterpret_cast<const void*>(v);
}

// Problems of a grouped phase's route table (the table is complete before
// the launch), clamped to the table's capacity.
__device__ __forceinline__ int route_problems(const int* route) {
  const int P = ld_field(route);
  return P < 0 ? 0 : (P > kRouteMaxProblems ? kRouteMaxProblems : P);
}

// Units of phase p: tiles x K units, times the problems of its route table
// for a grouped phase.
template <bool GROUPED>
__device__ __forceinline__ int phase_total(const Phase* phases, int p) {
  if (!GROUPED || !(ld_field(&phases[p].flags) & kPhaseGrouped)) return ld_field(&phases[p].total);
  const int* route = static_cast<const int*>(ld_field_ptr(reinterpret_cast<const void* const*>(&phases[p].route)));
  return route_problems(route) * ld_field(&phases[p].n_tiles) * ld_field(&phases[p].ku);
}

// Expert of problem pi; an id outside [0, experts) sets the device error
// word and reads expert 0 instead (the table comes from device memory and
// must never steer a weight read outside the stacked experts).
__device__ __forceinline__ int route_expert(const int* route, int pi, int experts) {
  const int e = ld_field(route + 2 + 2 * pi);
  if (e < 0 || e >= experts) {
    atomicExch(&g_device_error, kDevBadInput);
    return 0;
  }
  return e;
}

// CTA c's share of a phase of `total` units on a grid of G CTAs:
// [floor(c * total / G), floor((c + 1) * total / G)).
__device__ __forceinline__ int unit_begin(int c, int total, int grid) {
  return int((long long)c * total / grid);
}

// The CTA whose (non-empty) range holds unit u.
__device__ __forceinline__ int owner_of(int u, int total, int grid) {
  return int(((long long)(u + 1) * grid + total - 1) / total) - 1;
}

// Where a wait gave up (recorded once per launch in the workspace, read by
// tests and diagnostics; reset by the launch's last CTA): role code in the
// high byte, phase below.
enum WaitRole : int {
  kWhereDep = 1, kWhereGuard = 2, kWherePartial = 3, kWhereProducer = 4, kWhereMma = 5,
  kWhereDequant = 6, kWhereXFree = 7, kWhereAcc = 8,
};

__device__ __forceinline__ void record_timeout(int* words, int role, int phase, int d0 = 0,
                                               int d1 = 0, int d2 = 0, int d3 = 0) {
  atomicExch(&g_device_error, kDevWaitTimeout);
  if (atomicCAS(words + kWordWhere, 0, (role << 24) | (phase & 0xFFFFFF)) == 0) {
    atomicExch(words + kWordWhereCta, int(blockIdx.x));
    atomicExch(words + kWordDiag + 0, d0);
    atomicExch(words + kWordDiag + 1, d1);
    atomicExch(words + kWordDiag + 2, d2);
    atomicExch(words + kWordDiag + 3, d3);
  }
}

// Bounded mbarrier wait of the plan kernel: gives up at once when this CTA
// or the plan is aborting; on a time-out records where, and aborts both.
__device__ __forceinline__ bool plan_wait(uint64_t* bar, uint32_t parity, volatile int* cta_abort,
                                          volatile int* plan_abort, int* words, int role,
                                          int phase, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*cta_abort) return false;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*cta_abort) return false;
    if (*plan_abort) {
      *cta_abort = 1;
      return false;
    }
    if (globaltimer_ns() - t0 > limit_ns) {
      record_timeout(words, role, phase);
      *plan_abort = 1;
      *cta_abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void st_release(int* addr, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

// Spin until *addr >= target (acquire, gpu scope).  Gives up at once when
// the CTA or plan-wide abort word is set, or after limit_ns (then sets
// the device error word and both abort words).  Returns false on give-up.
__device__ __forceinline__ bool wait_counter(const int* addr, int target, volatile int* cta_abort,
                                             volatile int* plan_abort, int* words, int role,
                                             int phase, unsigned long long limit_ns) {
  if (ld_acquire(addr) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    __nanosleep(32);
    if (ld_acquire(addr) >= target) return true;
    if (*cta_abort) return false;
    if (*plan_abort) {
      *cta_abort = 1;
      return false;
    }
    if (globaltimer_ns() - t0 > limit_ns) {
      record_timeout(words, role, phase, target, ld_acquire(addr), int(addr - words));
      *plan_abort = 1;
      *cta_abort = 1;
      return false;
    }
  }
}

// Vote of the 128 epilogue threads (named_bar_and reconverges each warp
// first: lanes may arrive from different iterations of their own waits).
__device__ __forceinline__ bool epi_all(bool pred) { return named_bar_and(BAR_ID_EPI, 128, pred); }

template <int MT, bool GROUPED>
__global__ void __launch_bounds__(NUM_THREADS, 1) qmm_plan_kernel(const __grid_constant__ RunParams rp) {
  using C = Cfg<MT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BARS);
  uint64_t* full = bars;                       // [NSTAGE] unit block landed
  uint64_t* empty = full + C::NSTAGE;             // [NSTAGE] block read by the dequant warps
  uint64_t* afull = empty + C::NSTAGE;            // [NASLOT] TMEM A slot written
  uint64_t* aempty = afull + C::NASLOT;        // [NASLOT] TMEM A slot read by the MMAs
  uint64_t* xfull = aempty + C::NASLOT;        // [XS] x slot landed (TMA)
  uint64_t* xfree = xfull + C::XS;             // [XS] x slot read by all MMA warps
  uint64_t* accfull = xfree + C::XS;           // [NACCBUF]
  uint64_t* accempty = accfull + C::NACCBUF;   // [NACCBUF]
  uint64_t* drained = accempty + C::NACCBUF;   // [NUM_MMA_WARPS] an MMA warp's last ops done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + NUM_MMA_WARPS);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 2);
  volatile int* plan_abort = reinterpret_cast<volatile int*>(rp.words + kWordAbort);
  int* const words = rp.words;
  const unsigned long long limit_ns = rp.wait_limit_ns;
  auto wait = [abort_word, plan_abort, words, limit_ns](uint64_t* bar, uint32_t parity, int role,
                                                        int phase) {
    return plan_wait(bar, parity, abort_word, plan_abort, words, role, phase, limit_ns);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int G = gridDim.x;
  const int P = rp.n_phases;
  const Phase* phases = rp.phases;

  if (threadIdx.x == 0) {
    *abort_word = 0;
    for (int i = 0; i < C::NSTAGE; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4 * NDG);
    }
    for (int i = 0; i < C::NASLOT; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], C::NSLICE);
    }
    for (int i = 0; i < C::XS; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xfree[i], NUM_MMA_WARPS);
    }
    for (int i = 0; i < C::NACCBUF; ++i) {
      mbar_init(&accfull[i], NUM_MMA_WARPS);
      mbar_init(&accempty[i], 4);
    }
    for (int i = 0; i < NUM_MMA_WARPS; ++i) mbar_init(&drained[i], 1);
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

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------ producer
    // One bulk copy per unit into the NSTAGE ring; waits only for the
    // dequant warps to release a stage, never for another CTA.  (Prefetching
    // blocks further ahead into L2 was measured to gain nothing.)
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int it = 0;
      int n_total = phase_total<GROUPED>(phases, 0);
      const uint8_t* n_w = static_cast<const uint8_t*>(ld_field_ptr(reinterpret_cast<const void* const*>(&phases[0].w)));
      for (int p = 0; p < P && !*abort_word; ++p) {
        const int total = n_total;
        const uint8_t* w = n_w;
        if (p + 1 < P) {
          n_total = phase_total<GROUPED>(phases, p + 1);
          n_w = static_cast<const uint8_t*>(ld_field_ptr(reinterpret_cast<const void* const*>(&phases[p + 1].w)));
        }
        const int u0 = unit_begin(cta, total, G), u1 = unit_begin(cta + 1, total, G);
        const bool grouped = GROUPED && (ld_field(&phases[p].flags) & kPhaseGrouped) != 0;
        int g_nt = 0, g_ku = 1, g_ex = 1, last_pi = -1, e = 0;
        const int* route = nullptr;
        if (grouped) {
          g_nt = ld_field(&phases[p].n_tiles);
          g_ku = ld_field(&phases[p].ku);
          g_ex = ld_field(&phases[p].experts);
          route = static_cast<const int*>(ld_field_ptr(reinterpret_cast<const void* const*>(&phases[p].route)));
        }
        const uint8_t* src = w + size_t(u0) * BLK_BYTES;
        for (int u = u0; u < u1; ++u, ++it, src += BLK_BYTES) {
          if (grouped) {
            // unit u = (problem, tile, K unit): the problem's expert's block
            const int tt = u / g_ku, pi = tt / g_nt;
            if (pi != last_pi) {
              e = route_expert(route, pi, g_ex);
              last_pi = pi;
            }
            src = w + (size_t(e) * g_nt + (tt - pi * g_nt)) * g_ku * BLK_BYTES + size_t(u - tt * g_ku) * BLK_BYTES;
          }
          const int s = it % C::NSTAGE;
          if (!wait(&empty[s], ((it / C::NSTAGE) & 1) ^ 1, kWhereProducer, p)) break;
          mbar_arrive_expect_tx(&full[s], BLK_BYTES);
          bulk_load_hint(smem_u32(smem + s * BLK_BYTES), src, BLK_BYTES, &full[s], pol);
        }
      }
    }
    __syncwarp();
  } else if (warp < WARP_DQ0) {
    // ------------------------------------------------------------ MMA issuers
    // Warp j = a * NSLICE + sl issues the MMAs of sub-blocks a, a + NACC, ...
    // of every unit for token columns [sl * SLICE_N, (sl + 1) * SLICE_N) of
    // accumulator a; one accumulator segment per (phase, tile) part.  x
    // arrives in NCH chunks per unit; a chunk's slot is released once every
    // MMA warp's MMAs that read it completed.
    const int j = warp - WARP_MMA0;
    const int a_idx = j / C::NSLICE, sl = j % C::NSLICE;
    constexpr uint32_t idesc = make_idesc_16(BN, C::SLICE_N, false);
    const uint64_t ring_desc =
        make_sw128_desc(smem_u32(smem + C::OFF_XRING + sl * C::SLICE_N * 128));
    constexpr uint64_t kChunkDesc = uint64_t(C::XCHUNK_BYTES >> 4);
    constexpr uint64_t kBlkDesc = uint64_t(C::XBLK_BYTES >> 4);
    {
      int it = 0, acc_it = 0;
      uint32_t buf = 0;
      int n_total = phase_total<GROUPED>(phases, 0), n_ku = ld_field(&phases[0].ku);
      for (int p = 0; p < P; ++p) {
        const int total = n_total, ku = n_ku;
        if (p + 1 < P) {
          n_total = phase_total<GROUPED>(phases, p + 1);
          n_ku = ld_field(&phases[p + 1].ku);
        }
        const int u0 = unit_begin(cta, total, G), u1 = unit_begin(cta + 1, total, G);
        int kb = u0 % ku;
        for (int u = u0; u < u1; ++u, ++it, kb = (kb + 1 == ku) ? 0 : kb + 1) {
          const bool seg_start = (u == u0) || (kb == 0);
          const bool seg_end = (u == u1 - 1) || (kb == ku - 1);
          if (seg_start) {
            buf = acc_it % C::NACCBUF;
            wait(&accempty[buf], ((acc_it / C::NACCBUF) & 1) ^ 1, kWhereMma, p);
          }
          const uint32_t d_tmem =
              tmem_base + C::ACC_COL0 + buf * C::ACC_COLS + a_idx * MT + sl * C::SLICE_N;
          uint32_t acc0 = seg_start ? 0u : 1u;
#pragma unroll
          for (int ch = 0; ch < C::NCH; ++ch) {
            const int xseq = it * C::NCH + ch;
            const int xs = xseq % C::XS;
            wait(&xfull[xs], (xseq / C::XS) & 1, kWhereMma, p);
            const uint64_t chunk_desc = ring_desc + kChunkDesc * xs;
#pragma unroll
            for (int i = 0; i < C::XCH / C::NACC; ++i) {
              const int sbc = a_idx + i * C::NACC;       // sub-block within the chunk
              const int g = it * NSUB + ch * C::XCH + sbc;
              const int slot = g % C::NASLOT;
              wait(&afull[slot], (g / C::NASLOT) & 1, kWhereMma, p);
              tc_fence_after();
              if (!*abort_word) {
                const uint32_t a_tmem = tmem_base + slot * A_COLS;
                const uint64_t bdesc = chunk_desc + kBlkDesc * sbc;
                mma_bf16_ts_warp(d_tmem, a_tmem, bdesc, idesc, acc0);
                mma_bf16_ts_warp(d_tmem, a_tmem + 8, bdesc + 2, idesc, 1u);
                mma_bf16_ts_warp(d_tmem, a_tmem + 16, bdesc + 4, idesc, 1u);
                mma_bf16_ts_warp(d_tmem, a_tmem + 24, bdesc + 6, idesc, 1u);
              }
              acc0 = 1u;
              tc_commit_warp(&aempty[slot]);
            }
            if constexpr (!C::kXReleaseByA) tc_commit_warp(&xfree[xs]);
          }
          if (seg_end) {
            tc_commit_warp(&accfull[buf]);
            ++acc_it;
          }
        }
      }
    }
    // TMEM is freed only after this warp's MMAs completed.  On the normal
    // path the epilogue already waited for them; after an abort some may
    // still run, so wait (bounded, whatever the abort words say).
    tc_commit_warp(&drained[j]);
    mbar_wait(&drained[j], 0);
  } else if (warp < WARP_EPI0) {
    // ------------------------------------------------------------ dequant
    const int dw = warp - WARP_DQ0;
    const int grp = dw >> 2;               // sub-blocks grp + NDG * jj of every unit
    const int quad = warp & 3;             // TMEM lane quadrant
    const int r = quad * 32 + lane;        // output row within the tile
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    int it = 0;
    int n_total = phase_total<GROUPED>(phases, 0), n_flags = ld_field(&phases[0].flags);
    for (int p = 0; p < P; ++p) {
      const int total = n_total;
      const bool subn = (n_flags & kPhaseSubnormal) != 0;
      if (p + 1 < P) {
        n_total = phase_total<GROUPED>(phases, p + 1);
        n_flags = ld_field(&phases[p + 1].flags);
      }
      const int u0 = unit_begin(cta, total, G), u1 = unit_begin(cta + 1, total, G);
      for (int u = u0; u < u1; ++u, ++it) {
        const int s = it % C::NSTAGE;
        wait(&full[s], (it / C::NSTAGE) & 1, kWhereDequant, p);
        const uint32_t st = smem_u32(smem + s * BLK_BYTES);
        // this thread's packed words (SPG sub-blocks x 8 words) and its
        // scales / biases, then the stage goes back to the producer.  Group
        // grp converts sub-blocks sb = grp + NDG * jj; sub-block sb's scale
        // and bias are half sb / 4 of record sb % 4.
        uint2 sbw[RPG];
#pragma unroll
        for (int q = 0; q < RPG; ++q)
          sbw[q] = ld_shared_v2(st + PACK_BYTES + uint32_t((grp + NDG * q) * BN + r) * 8u);
        uint4 qv[SPG][2];
#pragma unroll
        for (int jj = 0; jj < SPG; ++jj)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            qv[jj][h] = ld_shared_v4(st + uint32_t(((grp + NDG * jj) * 2 + h) * BN + r) * 16u);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        int slots[SPG];
#pragma unroll
        for (int jj = 0; jj < SPG; ++jj) {
          const int g = it * NSUB + grp + NDG * jj;
          const int slot = g % C::NASLOT;
          slots[jj] = slot;
          wait(&aempty[slot], ((g / C::NASLOT) & 1) ^ 1, kWhereDequant, p);
          tc_fence_after();
          const uint2 rec = sbw[jj % RPG];
          const uint32_t sel = (jj / RPG) ? 0x3232u : 0x1010u;
          const uint32_t s2 = __byte_perm(rec.x, 0, sel);
          const uint32_t b2 = __byte_perm(rec.y, 0, sel);
          uint32_t w[32];
          if (subn) {
            const uint32_t s_hi = bf16x2_mul(s2, 0x3D803D80u);  // * 2^-4
            dequant8_subn(qv[jj][0].x, s2, s_hi, b2, &w[0]);
            dequant8_subn(qv[jj][0].y, s2, s_hi, b2, &w[4]);
            dequant8_subn(qv[jj][0].z, s2, s_hi, b2, &w[8]);
            dequant8_subn(qv[jj][0].w, s2, s_hi, b2, &w[12]);
            dequant8_subn(qv[jj][1].x, s2, s_hi, b2, &w[16]);
            dequant8_subn(qv[jj][1].y, s2, s_hi, b2, &w[20]);
            dequant8_subn(qv[jj][1].z, s2, s_hi, b2, &w[24]);
            dequant8_subn(qv[jj][1].w, s2, s_hi, b2, &w[28]);
          } else {
            dequant8_magic(qv[jj][0].x, s2, b2, &w[0]);
            dequant8_magic(qv[jj][0].y, s2, b2, &w[4]);
            dequant8_magic(qv[jj][0].z, s2, b2, &w[8]);
            dequant8_magic(qv[jj][0].w, s2, b2, &w[12]);
            dequant8_magic(qv[jj][1].x, s2, b2, &w[16]);
            dequant8_magic(qv[jj][1].y, s2, b2, &w[20]);
            dequant8_magic(qv[jj][1].z, s2, b2, &w[24]);
            dequant8_magic(qv[jj][1].w, s2, b2, &w[28]);
          }
          tmem_st_32x32b_x32(lane_base + slot * A_COLS, w);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int jj = 0; jj < SPG; ++jj) mbar_arrive(&afull[slots[jj]]);
        }
      }
    }
  } else if (warp == WARP_X) {
    // ------------------------------------------------------------ x loads
    // x for every unit of this CTA, in order, in NCH chunks per unit into the
    // XS-slot ring: waits only for the MMAs to free a slot and, for a phase
    // with a dependency, for every CTA to have signalled that phase complete
    // (this CTA's own epilogues of it need no x beyond what is already
    // loaded, so the wait always ends).
    if (lane == 0) {
      int seq = 0;
      bool ok = true;
      for (int p = 0; ok && p < P; ++p) {
        const Phase& ph = phases[p];
        const int total = phase_total<GROUPED>(phases, p), ku = ld_field(&ph.ku), dep = ld_field(&ph.dep);
        const int u0 = unit_begin(cta, total, G), u1 = unit_begin(cta + 1, total, G);
        if (u0 == u1) continue;
        const bool grouped = GROUPED && (ld_field(&ph.flags) & kPhaseGrouped) != 0;
        const int g_nt = ld_field(&ph.n_tiles);
        const int* route =
            grouped ? static_cast<const int*>(ld_field_ptr(reinterpret_cast<const void* const*>(&ph.route))) : nullptr;
        // the x tensor map was written into global memory by a host copy:
        // order that write before the TMA unit's reads of the map
        asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(
                         reinterpret_cast<uint64_t>(&ph.tm_x))
                     : "memory");
        // a grouped phase reading an earlier grouped phase's rows waits per
        // problem (that problem's tiles of the earlier phase stored)
        const int wslot = grouped ? (ld_field(&ph.flags) >> kWaitShift) & 0xFF : 0;
        const int dep_nt = wslot ? ld_field(&phases[dep].n_tiles) : 0;
        if (dep >= 0 && wslot == 0) {
          // a dependency wait spans the whole earlier phase, so it runs twice
          // the limit: a stall inside that phase is then reported by the wait
          // that sees it first-hand (split-K partial, guard, pipeline) rather
          // than by this downstream wait
          if (!wait_counter(rp.words + dep, G, abort_word, plan_abort, words, kWhereDep, p, 2 * limit_ns)) break;
          fence_proxy_async_global();   // x rows written by other CTAs' stores
        }
        int last_pi = -1, row0 = 0;
        for (int u = u0; ok && u < u1; ++u) {
          const int k0 = (u % ku) * UNIT_K;
          // x rows of a grouped phase: the unit's problem's sorted rows
          if (grouped && (u / ku) / g_nt != last_pi) {
            last_pi = (u / ku) / g_nt;
            row0 = ld_field(route + 1 + 2 * last_pi);
            if (wslot) {
              if (!wait_counter(rp.words + kWordProblem + (wslot - 1) * kRouteMaxProblems + last_pi, dep_nt,
                                abort_word, plan_abort, words, kWhereDep, p, 2 * limit_ns)) {
                ok = false;
                break;
              }
              fence_proxy_async_global();   // x rows written by other CTAs' stores
            }
          }
#pragma unroll 1
          for (int ch = 0; ch < C::NCH; ++ch, ++seq) {
            const int xs = seq % C::XS;
            if (seq >= C::XS) {
              bool freed;
              if constexpr (C::kXReleaseByA) {
                // the slot's previous chunk: its last sub-block's A slot released
                const int qq = seq - C::XS;
                const int g = (qq / C::NCH) * NSUB + (qq % C::NCH) * C::XCH + C::XCH - 1;
                freed = wait(&aempty[g % C::NASLOT], (g / C::NASLOT) & 1, kWhereXFree, p);
              } else {
                freed = wait(&xfree[xs], ((seq / C::XS) - 1) & 1, kWhereXFree, p);
              }
              if (!freed) {
                ok = false;
                break;
              }
            }
            uint8_t* dst = smem + C::OFF_XRING + xs * C::XCHUNK_BYTES;
            mbar_arrive_expect_tx(&xfull[xs], C::XCHUNK_BYTES);
#pragma unroll
            for (int b = 0; b < C::XCH; ++b)
              tma_load_2d(dst + b * C::XBLK_BYTES, &ph.tm_x, &xfull[xs], k0 + (ch * C::XCH + b) * GS, row0);
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------ epilogue + split-K + phase signals
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int et = threadIdx.x - WARP_EPI0 * 32;   // 0..127
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    int* const ready = rp.words + kWordReady;
    int* const consumed = rp.words + kWordConsumed;

    int acc_it = 0;
    int lastw[kSlotPhases] = {0, 0, 0, 0};  // phase + 1 of this CTA's last partial per slot
    bool ok = true;
    int n_total = phase_total<GROUPED>(phases, 0), n_ku = ld_field(&phases[0].ku);
    for (int p = 0; ok && p < P; ++p) {
      const Phase& ph = phases[p];
      const int total = n_total, ku = n_ku;
      if (p + 1 < P) {
        n_total = phase_total<GROUPED>(phases, p + 1);
        n_ku = ld_field(&phases[p + 1].ku);
      }
      const int u0 = unit_begin(cta, total, G), u1 = unit_begin(cta + 1, total, G);
      const int par = p % kSlotPhases;
      if (u0 < u1) {
        const int M = ph.M, N = ph.N, ldy = ph.ldy;
        const bool silu = (ph.flags & kPhaseSilu) != 0;
        const bool grouped = GROUPED && (ph.flags & kPhaseGrouped) != 0;
        const bool scatter = GROUPED && (ph.flags & kPhaseScatter) != 0;
        const int g_nt = ph.n_tiles;
        const int* const route = ph.route;
        const int sig_slot = grouped ? (ph.flags >> kSignalShift) & 0xFF : 0;
        const bool vec = (ph.flags & kVecStore) != 0;
        uint16_t* const y = ph.y;
        const int t_first = u0 / ku, t_last = (u1 - 1) / ku;
        for (int t = t_first; t <= t_last; ++t) {
          const int kb0 = (t == t_first) ? (u0 - t * ku) : 0;
          const int kb1 = (t == t_last) ? (u1 - t * ku) : ku;
          const bool full_tile = (kb0 == 0 && kb1 == ku);
          const int c_lo = full_tile ? cta : owner_of(t * ku, total, G);
          const bool collect = !full_tile && cta == c_lo;
          const int c_hi = collect ? owner_of(t * ku + ku - 1, total, G) : c_lo;
          if (!full_tile && cta != c_lo) {
            // contributor: the consumer of its previous partial in this slot
            // must have read it before the slot is refilled (almost always
            // already true)
            bool gok = true;
            if (et == 0 && lastw[par] > 0 && ld_acquire(consumed + kSlotPhases * cta + par) < lastw[par])
              gok = wait_counter(consumed + kSlotPhases * cta + par, lastw[par], abort_word, plan_abort, words,
                                 kWhereGuard, p, limit_ns);
            if (!epi_all(gok && !*abort_word)) {
              ok = false;
              break;
            }
          }
          // c_lo: the contributors computed this tile's other parts first in
          // their ranges, so their partials are ready (or nearly) while this
          // CTA's own MMAs for the tile still run.  They are summed in CTA
          // order; with one epilogue pass (MT <= 32) that happens here and
          // each slot is marked read at once, otherwise pass by pass below.
          float psum[C::kEarlyPartials ? MT : 1];
          if (collect) {
            if constexpr (C::kEarlyPartials) {
#pragma unroll
              for (int m = 0; m < MT; ++m) psum[m] = 0.f;
            }
            if constexpr (C::kEarlyPartials) {
              // 16-row tiles (one or two contributors, usually): each
              // contributor's stamp, its partial summed in CTA order, then
              // its slot released
              for (int c = c_lo + 1; ok && c <= c_hi; ++c) {
                if (unit_begin(c, total, G) == unit_begin(c + 1, total, G)) continue;
                const bool pok = wait_counter(ready + kSlotPhases * c + par, p + 1, abort_word, plan_abort,
                                              words, kWherePartial, p, limit_ns);
                if (pok) {
                  if constexpr (C::kFragEpi) {
                    const float* slot = rp.partials + size_t(kSlotPhases * c + par) * MT * BN + et * 16;
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                      const float4 q4 = ld_relaxed_v4(slot + 4 * v);
                      psum[4 * v] += q4.x;
                      psum[4 * v + 1] += q4.y;
                      psum[4 * v + 2] += q4.z;
                      psum[4 * v + 3] += q4.w;
                    }
                  } else {
                    const uint32_t* slot =
                        reinterpret_cast<const uint32_t*>(rp.partials) + size_t(kSlotPhases * c + par) * MT * BN;
#pragma unroll
                    for (int m = 0; m < MT; ++m) psum[m] += __uint_as_float(ld_relaxed_u32(slot + m * BN + r));
                  }
                }
                // every thread has read the slot: its contributor may refill it
                if (!epi_all(pok && !*abort_word)) {
                  ok = false;
                  break;
                }
                if (et == 0) st_release(consumed + kSlotPhases * c + par, p + 1);
              }
            } else {
              // 32+ rows (partials summed pass by pass below): every
              // contributor's stamp awaited by its own epilogue thread
              // (acquire), then one barrier makes all of them visible to
              // every thread (acquire + bar.sync) instead of one wait and
              // barrier per contributor in turn
              bool pok = true;
              for (int j = et; j < c_hi - c_lo; j += 128) {
                const int c = c_lo + 1 + j;
                if (unit_begin(c, total, G) != unit_begin(c + 1, total, G))
                  pok = pok && wait_counter(ready + kSlotPhases * c + par, p + 1, abort_word, plan_abort, words,
                                            kWherePartial, p, limit_ns);
              }
              if (!epi_all(pok && !*abort_word)) ok = false;
            }
            if (!ok) break;
          }
          const uint32_t buf = acc_it % C::NACCBUF;
          const bool got = wait(&accfull[buf], (acc_it / C::NACCBUF) & 1, kWhereAcc, p);
          if (!epi_all(got && !*abort_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // output columns of the tile; a grouped phase's tile t is tile
          // t % n_tiles of problem t / n_tiles, whose rows are the problem's
          // sorted rows (scattered to pair rows through the route table)
          int t_loc = t, row0 = 0, rows = M;
          if (grouped) {
            // rows [row0, row0 + rows) of the phase's M rows, at most one tile
            const int pi = t / g_nt;
            t_loc = t - pi * g_nt;
            row0 = ld_field(route + 1 + 2 * pi);
            rows = ld_field(route + 3 + 2 * pi) - row0;
            if (row0 < 0 || row0 >= M) rows = 0;
            rows = rows < 0 ? 0 : (rows > MT ? MT : rows);
            rows = rows > M - row0 ? M - row0 : rows;
          }
          // output row of tile row m (< rows): the sorted row, or with a
          // scatter the pair row the route table maps it to (one past the
          // phase's rows when the table holds an out-of-range row: skipped)
          auto out_row = [&](int m) -> size_t {
            if (!scatter) return size_t(row0 + m);
            const int o = ld_field(route + kRouteRowMap + row0 + m);
            return size_t(o >= 0 && o < M ? o : M);
          };
          if constexpr (!C::kFragEpi) {
          // 16-token tiles: one thread per output column, one store per value
          const int n = t_loc * BN + r;
          uint32_t* const mine = reinterpret_cast<uint32_t*>(rp.partials) + size_t(kSlotPhases * cta + par) * MT * BN;
#pragma unroll 1
          for (int c0 = 0; c0 < MT; c0 += C::EC) {
            // c_lo with several passes: the contributors' partials of this
            // pass, summed in CTA order (two contributors' loads in flight
            // at a time), before the accumulator columns are read
            float ps[C::EC];
            if constexpr (!C::kEarlyPartials) {
              if (collect) {
#pragma unroll
                for (int m = 0; m < C::EC; ++m) ps[m] = 0.f;
                for (int c = c_lo + 1; c <= c_hi; ++c) {
                  if (unit_begin(c, total, G) == unit_begin(c + 1, total, G)) continue;
                  const uint32_t* sa = reinterpret_cast<const uint32_t*>(rp.partials) +
                                       size_t(kSlotPhases * c + par) * MT * BN + size_t(c0) * BN + r;
#pragma unroll
                  for (int m = 0; m < C::EC; ++m) ps[m] += __uint_as_float(ld_relaxed_u32(sa + m * BN));
                }
              }
            }
            float acc[C::EC];
            {
              uint32_t rr[16];
#pragma unroll
              for (int c = 0; c < C::EC; c += 16) {
#pragma unroll
                for (int a = 0; a < C::NACC; ++a) {
                  tmem_ld_32x32b_x16(lane_base + C::ACC_COL0 + buf * C::ACC_COLS + a * MT + c0 + c, rr);
                  tmem_ld_wait();
#pragma unroll
                  for (int i = 0; i < 16; ++i)
                    acc[c + i] = (a == 0) ? __uint_as_float(rr[i]) : acc[c + i] + __uint_as_float(rr[i]);
                }
              }
            }
            if (c0 + C::EC == MT) {
              // the accumulator buffer is read: the MMAs may reuse it
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&accempty[buf]);
            }
            if (!full_tile && cta != c_lo) {
              // contributor: this pass of its partial into its own slot
#pragma unroll
              for (int m = 0; m < C::EC; ++m)
                st_relaxed_u32(mine + (c0 + m) * BN + r, __float_as_uint(acc[m]));
              continue;
            }
            if (collect) {
              // c_lo: its own accumulator plus the contributors' partial sum
              if constexpr (C::kEarlyPartials) {
#pragma unroll
                for (int m = 0; m < C::EC; ++m) acc[m] += psum[m];
              } else {
#pragma unroll
                for (int m = 0; m < C::EC; ++m) acc[m] += ps[m];
              }
            }
            if (n >= N) continue;
            if (silu) {
              // rows interleaved in blocks of 32 (16 gate, then the 16 up rows
              // of the same outputs): lanes 0-15 hold gate, 16-31 up.  Each
              // lane swaps its rounded values with its partner (lane ^ 16);
              // lanes 0-15 then finish the even tokens and 16-31 the odd ones,
              // so all 32 lanes run the SiLU and its steps overlap across tokens.
              const int hcol = (n >> 5) * 16 + (lane & 15);
              const bool lo = lane < 16;
              uint32_t own[C::EC], oth[C::EC];
#pragma unroll
              for (int m = 0; m < C::EC; ++m) own[m] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[m]));
#pragma unroll
              for (int m = 0; m < C::EC; ++m) oth[m] = __shfl_xor_sync(0xffffffffu, own[m], 16);
#pragma unroll
              for (int mp = 0; mp < C::EC / 2; ++mp) {
                const int m = 2 * mp + (lo ? 0 : 1);
                const uint32_t gbits = lo ? own[2 * mp] : oth[2 * mp + 1];
                const uint32_t ubits = lo ? oth[2 * mp] : own[2 * mp + 1];
                const uint16_t h = silu_mul_bits<false>(uint16_t(gbits), uint16_t(ubits));
                if (c0 + m < rows) {
                  const size_t orow = out_row(c0 + m);
                  if (orow < size_t(M)) y[orow * ldy + hcol] = h;
                }
              }
            } else {
#pragma unroll
              for (int m = 0; m < C::EC; ++m) {
                if (c0 + m < rows) {
                  const size_t orow = out_row(c0 + m);
                  if (orow < size_t(M)) y[orow * ldy + n] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[m]));
                }
              }
            }
          }
          } else {
          // Pass layout (16 tokens): accumulator lanes are output columns,
          // TMEM columns tokens.  Thread t of quadrant warp q holds acc[8h + j]
          // = column 32q + 16h + fa + 8((j >> 1) & 1), token tb + (j & 1) +
          // 8(j >> 2) of the pass (fa = t / 4, tb = 2(t % 4)): the fragment
          // layout of the 16x256b TMEM loads, which stmatrix.trans turns into
          // token rows for 16-byte stores.  Split-K partials keep the same
          // per-thread assignment: 16 contiguous floats per thread and pass.
          const int fa = lane >> 2, tb = 2 * (lane & 3);
          const int n_q = t_loc * BN + 32 * quad;    // first output column of this warp
          float* const mine = rp.partials + size_t(kSlotPhases * cta + par) * MT * BN + et * 16;
          const uint32_t stage_w = smem_u32(smem + C::OFF_STAGE) + uint32_t(quad * C::STAGE_WARP_BYTES);
#pragma unroll 1
          for (int c0 = 0; c0 < MT; c0 += C::EC) {
            // c_lo with several passes: the contributors' partials of this
            // pass, summed in CTA order, before the accumulator is read
            float ps[C::EC];
            if constexpr (!C::kEarlyPartials) {
              if (collect) {
#pragma unroll
                for (int m = 0; m < C::EC; ++m) ps[m] = 0.f;
                for (int c = c_lo + 1; c <= c_hi; ++c) {
                  if (unit_begin(c, total, G) == unit_begin(c + 1, total, G)) continue;
                  const float* sa = rp.partials + size_t(kSlotPhases * c + par) * MT * BN + size_t(c0) * BN + et * 16;
#pragma unroll
                  for (int v = 0; v < 4; ++v) {
                    const float4 q4 = ld_relaxed_v4(sa + 4 * v);
                    ps[4 * v] += q4.x;
                    ps[4 * v + 1] += q4.y;
                    ps[4 * v + 2] += q4.z;
                    ps[4 * v + 3] += q4.w;
                  }
                }
              }
            }
            float acc[C::EC];
            {
              uint32_t ra[8], rb[8];
#pragma unroll
              for (int a = 0; a < C::NACC; ++a) {
                const uint32_t col = uint32_t(C::ACC_COL0 + buf * C::ACC_COLS + a * MT + c0);
                tmem_ld_16x256b_x2(lane_base + col, ra);
                tmem_ld_16x256b_x2(lane_base + (16u << 16) + col, rb);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  acc[i] = (a == 0) ? __uint_as_float(ra[i]) : acc[i] + __uint_as_float(ra[i]);
                  acc[8 + i] = (a == 0) ? __uint_as_float(rb[i]) : acc[8 + i] + __uint_as_float(rb[i]);
                }
              }
            }
            if (c0 + C::EC == MT) {
              // the accumulator buffer is read: the MMAs may reuse it
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&accempty[buf]);
            }
            if (!full_tile && cta != c_lo) {
              // contributor: this pass of its partial into its own slot
#pragma unroll
              for (int v = 0; v < 4; ++v)
                st_relaxed_v4(mine + size_t(c0) * BN + 4 * v, acc[4 * v], acc[4 * v + 1], acc[4 * v + 2],
                              acc[4 * v + 3]);
              continue;
            }
            if (collect) {
              // c_lo: its own accumulator plus the contributors' partial sum
              if constexpr (C::kEarlyPartials) {
#pragma unroll
                for (int m = 0; m < C::EC; ++m) acc[m] += psum[m];
              } else {
#pragma unroll
                for (int m = 0; m < C::EC; ++m) acc[m] += ps[m];
              }
            }
            const int nrows = min(C::EC, rows - c0);
            if (silu) {
              // columns in blocks of 32 (16 gate, then the 16 up columns of
              // the same outputs): this warp's block is quadrant q, so each
              // thread holds the gate (h = 0) and up (h = 1) values of its
              // outputs fa, fa + 8 for its four tokens
              const int hq = (t_loc * 4 + quad) * 16;   // first output of this warp
              uint32_t hv[8];
#pragma unroll
              for (int j = 0; j < 8; ++j)
                hv[j] = silu_mul_bits<false>(__bfloat16_as_ushort(__float2bfloat16_rn(acc[j])),
                                             __bfloat16_as_ushort(__float2bfloat16_rn(acc[8 + j])));
              if (vec) {
                const int i = lane >> 3, rho = lane & 7;
                stmatrix_x4_trans(stage_w + uint32_t(((i >> 1) * 8 + rho) * C::STAGE_ROW_BYTES + (i & 1) * 16),
                                  hv[0] | (hv[1] << 16), hv[2] | (hv[3] << 16), hv[4] | (hv[5] << 16),
                                  hv[6] | (hv[7] << 16));
                __syncwarp();
                const int m = lane >> 1, ch = lane & 1;
                if (m < nrows && n_q < N) {
                  const size_t orow = out_row(c0 + m);
                  if (orow < size_t(M))
                    *reinterpret_cast<uint4*>(y + orow * ldy + hq + ch * 8) =
                        ld_shared_v4(stage_w + uint32_t(m * C::STAGE_ROW_BYTES + ch * 16));
                }
                __syncwarp();
              } else if (n_q < N) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int k = tb + (j & 1) + 8 * (j >> 2);
                  if (k < nrows) {
                    const size_t orow = out_row(c0 + k);
                    if (orow < size_t(M)) y[orow * ldy + hq + fa + 8 * ((j >> 1) & 1)] = uint16_t(hv[j]);
                  }
                }
              }
            } else if (vec) {
              const int i = lane >> 3, rho = lane & 7;
#pragma unroll
              for (int h = 0; h < 2; ++h)
                stmatrix_x4_trans(
                    stage_w + uint32_t(((i >> 1) * 8 + rho) * C::STAGE_ROW_BYTES + (2 * h + (i & 1)) * 16),
                    pack_bf16(acc[8 * h], acc[8 * h + 1]), pack_bf16(acc[8 * h + 2], acc[8 * h + 3]),
                    pack_bf16(acc[8 * h + 4], acc[8 * h + 5]), pack_bf16(acc[8 * h + 6], acc[8 * h + 7]));
              __syncwarp();
              const int ch = lane & 3;
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int m = hh * 8 + (lane >> 2);
                if (m < nrows && n_q + ch * 8 < N) {
                  const size_t orow = out_row(c0 + m);
                  if (orow < size_t(M))
                    *reinterpret_cast<uint4*>(y + orow * ldy + n_q + ch * 8) =
                        ld_shared_v4(stage_w + uint32_t(m * C::STAGE_ROW_BYTES + ch * 16));
                }
              }
              __syncwarp();
            } else {
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int k = tb + (j & 1) + 8 * (j >> 2);
                  const int nn = n_q + 16 * h + fa + 8 * ((j >> 1) & 1);
                  if (k < nrows && nn < N) {
                    const size_t orow = out_row(c0 + k);
                    if (orow < size_t(M)) y[orow * ldy + nn] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[8 * h + j]));
                  }
                }
            }
          }
          }
          ++acc_it;
          if (!full_tile && cta != c_lo) {
            // the barrier orders every thread's partial stores before the
            // stamp's release (cumulativity)
            if (!epi_all(!*abort_word)) {
              ok = false;
              break;
            }
            // (a test can make one CTA withhold its partials: the consumer's
            // bounded wait then runs out and the plan winds down)
            if (et == 0 && cta != rp.skip_partial_cta) st_release(ready + kSlotPhases * cta + par, p + 1);
            lastw[par] = p + 1;
            continue;
          }
          if (!C::kEarlyPartials && !full_tile) {
            // every thread has read every contributor's slot: mark them read
            if (!epi_all(!*abort_word)) {
              ok = false;
              break;
            }
            if (et == 0)
              for (int c = c_lo + 1; c <= c_hi; ++c)
                if (unit_begin(c, total, G) != unit_begin(c + 1, total, G))
                  st_release(consumed + kSlotPhases * c + par, p + 1);
          }
          if (sig_slot > 0) {
            // the tile's final values are stored (the barrier orders every
            // thread's stores before the release): count it for its problem
            if (!epi_all(!*abort_word)) {
              ok = false;
              break;
            }
            if (et == 0)
              red_release_add(rp.words + kWordProblem + (sig_slot - 1) * kRouteMaxProblems + t / g_nt, 1);
          }
        }
      }
      if (!ok) break;
      // every final value of phase p this CTA owes is stored: signal it (the
      // barrier orders all 128 threads' stores before the release)
      if (!epi_all(!*abort_word)) {
        ok = false;
        break;
      }
      if (et == 0) red_release_add(rp.words + p, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_TMA) tmem_dealloc(tmem_base, TMEM_COLS);
  // The last CTA to leave zeroes the phase counters and slot counts for the
  // next launch (every other CTA is past its last use of them).
  if (threadIdx.x == 0) {
    __threadfence();
    *last_flag = (atomicAdd(rp.words + kWordExit, 1) == G - 1) ? 1 : 0;
  }
  __syncthreads();
  if (*last_flag) {
    __threadfence();
    for (int i = threadIdx.x; i < P; i += NUM_THREADS) rp.words[i] = 0;
    for (int i = threadIdx.x; i < 2 * kSlotPhases * kMaxGrid; i += NUM_THREADS) rp.words[kWordReady + i] = 0;
    for (int i = threadIdx.x; i < rp.prob_slots * kRouteMaxProblems; i += NUM_THREADS)
      rp.words[kWordProblem + i] = 0;
    if (threadIdx.x == 0) {
      rp.words[kWordAbort] = 0;
      rp.words[kWordExit] = 0;
    }
    // kWordWhere / kWordWhereCta stay set after a time-out for the host to
    // read (dfl_qmm_plan_last_timeout); the host clears them with the rest of
    // the workspace after a device error
  }
}

// MLX-packed int4 [N, K/8] + bf16 scales / biases [N, K/64] -> tiled blob.
// Work item i of a block: i < 2048 is the 16-byte nibble chunk (ch, r) at
// offset (ch * 128 + r) * 16 -- words w = 0..3 hold columns
// sb * 64 + h * 32 + 8w .. +8 of the unit (sb = ch / 2, h = ch % 2) in the
// pair-packed nibble order; i >= 2048 are two 8-byte scale/bias records
// (g, r) at PACK_BYTES + (g * 128 + r) * 8 = {s_g, s_g+4, b_g, b_g+4}.
__device__ __forceinline__ uint32_t pair_pack(uint32_t q) {
  uint32_t o = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    o |= ((q >> (8 * j)) & 0xFu) << (4 * j);
    o |= ((q >> (8 * j + 4)) & 0xFu) << (4 * (j + 4));
  }
  return o;
}

__device__ __forceinline__ uint16_t tiled_scale(uint16_t sv, bool subn) {
  if (!subn) return sv;
  float f = __bfloat162float(__ushort_as_bfloat16(sv));
  if (!(fabsf(f) < 0.03125f)) {   // also catches NaN / inf
    atomicExch(&g_device_error, kDevBadInput);
    return 0;
  }
  f = (f * 0x1p66f) * 0x1p67f;    // exact: a power-of-two scaling inside the range
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__global__ void repack_tiled_kernel(const uint32_t* __restrict__ wq, const uint16_t* __restrict__ sc,
                                    const uint16_t* __restrict__ bi, int N, int K, int ku,
                                    int subn, uint8_t* __restrict__ dst, long long n_items) {
  constexpr int PER_BLOCK = PACK_BYTES / 16 + SB_BYTES / 16;  // 2304
  const int kw = K / 8, kg = K / GS;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_items;
       i += (long long)gridDim.x * blockDim.x) {
    const long long blk = i / PER_BLOCK;
    const int e = int(i - blk * PER_BLOCK);
    const int t = int(blk / ku), kb = int(blk - (long long)t * ku);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (e < PACK_BYTES / 16) {
      const int ch = e / BN, r = e - ch * BN;
      const int n = t * BN + r;
      const int kcol0 = kb * UNIT_K + (ch >> 1) * GS + (ch & 1) * 32;
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int kc = kcol0 + 8 * q;
        w[q] = (n < N && kc < K) ? pair_pack(wq[(size_t)n * kw + kc / 8]) : 0u;
      }
      v = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      uint32_t rec[4];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int idx = 2 * (e - PACK_BYTES / 16) + half;   // record (g, r), 0..511
        const int g = idx / BN, r = idx - g * BN;
        const int n = t * BN + r;
        const int g0 = kb * NSUB + g, g1 = g0 + 4;
        uint16_t s0 = 0, s1 = 0, b0 = 0, b1 = 0;
        if (n < N) {
          if (g0 < kg) {
            s0 = tiled_scale(sc[(size_t)n * kg + g0], subn != 0);
            b0 = bi[(size_t)n * kg + g0];
          }
          if (g1 < kg) {
            s1 = tiled_scale(sc[(size_t)n * kg + g1], subn != 0);
            b1 = bi[(size_t)n * kg + g1];
          }
        }
        rec[2 * half] = uint32_t(s0) | (uint32_t(s1) << 16);
        rec[2 * half + 1] = uint32_t(b0) | (uint32_t(b1) << 16);
      }
      v = make_uint4(rec[0], rec[1], rec[2], rec[3]);
    }
    *reinterpret_cast<uint4*>(dst + blk * BLK_BYTES + size_t(e) * 16) = v;
  }
}

// ------------------------------------------------------------------ host
inline size_t tiled_bytes(int N, int K) {
  return size_t((N + BN - 1) / BN) * size_t((K + UNIT_K - 1) / UNIT_K) * BLK_BYTES;
}

inline size_t plan_bytes(int n) { return kHeaderBytes + size_t(n) * sizeof(Phase); }

inline size_t workspace_bytes(int mt, int grid) {
  return kCounterBytes + size_t(grid) * kSlotPhases * mt * BN * sizeof(float);
}

// GROUPED: the plan has grouped phases (route tables); plans without any run
// the variant compiled without that code.
template <int MT, bool GROUPED>
int launch(const Header& h, const void* plan_dev, void* ws, int dev, cudaStream_t stream) {
  using C = Cfg<MT>;
  static std::atomic<uint64_t> smem_done{0};
  int st = host::ensure_smem(qmm_plan_kernel<MT, GROUPED>, C::SMEM_BYTES, dev, smem_done);
  if (st != DFL_OK) return st;
  RunParams rp;
  rp.phases = reinterpret_cast<const Phase*>(static_cast<const uint8_t*>(plan_dev) + kHeaderBytes);
  rp.n_phases = h.n_phases;
  rp.skip_partial_cta = h.test_skip_partial_cta;
  rp.prob_slots = h.prob_slots;
  rp.wait_limit_ns = h.wait_limit_ns;
  rp.words = static_cast<int*>(ws);
  rp.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kCounterBytes);
  // CTAs wait on one another (phase counters, split-K partials): launched
  // cooperatively so that all of them are resident at once.
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(h.grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, qmm_plan_kernel<MT, GROUPED>, rp) != cudaSuccess) {
    cudaGetLastError();
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

inline int check_header(const void* plan_host, Header* out) {
  if (!plan_host) return DFL_ERR_NULL_POINTER;
  std::memcpy(out, plan_host, sizeof(Header));
  if (out->magic != kPlanMagic || out->version != kPlanVersion || out->n_phases < 1 ||
      out->n_phases > kMaxPhases ||
      (out->mt != 16 && out->mt != 32 && out->mt != 64 && out->mt != 128) || out->grid < 1 ||
      out->grid > kMaxGrid || out->wait_limit_ns == 0 || out->wait_limit_ns > kWaitLimitNs ||
      out->prob_slots < 0 || out->prob_slots > kMaxProblemSlots)
    return DFL_ERR_BAD_SHAPE;
  return DFL_OK;
}

}  // namespace plan
}  // namespace dfl

extern "C" size_t dfl_w4_tiled_bytes(int N, int K) {
  if (N < 1 || K < 64 || K % 64 != 0) return 0;
  return dfl::plan::tiled_bytes(N, K);
}

extern "C" int dfl_repack_w4_tiled(const uint32_t* w_q, const uint16_t* scales,
                                   const uint16_t* biases, int N, int K, int subnormal, void* dst,
                                   size_t dst_bytes, void* stream) {
  using namespace dfl;
  if (N < 1 || K < 64 || K % 64 != 0 || N > (1 << 24)) return DFL_ERR_BAD_SHAPE;
  if (!w_q || !scales || !biases || !dst) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(w_q, 4) || !host::aligned(scales, 2) || !host::aligned(biases, 2) ||
      !host::aligned(dst, 16))
    return DFL_ERR_MISALIGNED;
  if (dst_bytes < plan::tiled_bytes(N, K)) return DFL_ERR_WORKSPACE;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  const int ku = (K + plan::UNIT_K - 1) / plan::UNIT_K;
  const long long n_items =
      (long long)((N + plan::BN - 1) / plan::BN) * ku * (plan::PACK_BYTES / 16 + plan::SB_BYTES / 16);
  const long long want = (n_items + 255) / 256;
  const int blocks = int(want < (long long)sms * 16 ? want : (long long)sms * 16);
  plan::repack_tiled_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      w_q, scales, biases, N, K, ku, subnormal ? 1 : 0, static_cast<uint8_t*>(dst), n_items);
  return host::launch_status();
}

extern "C" size_t dfl_qmm_plan_bytes(int n_phases) {
  if (n_phases < 1 || n_phases > dfl::plan::kMaxPhases) return 0;
  return dfl::plan::plan_bytes(n_phases);
}

extern "C" int dfl_qmm_plan_encode(const dfl_qmm_phase* phases, int n_phases, void* plan_host,
                                   size_t plan_bytes) {
  using namespace dfl;
  using namespace dfl::plan;
  if (n_phases < 1 || n_phases > kMaxPhases) return DFL_ERR_BAD_SHAPE;
  if (!phases || !plan_host) return DFL_ERR_NULL_POINTER;
  if (plan_bytes < plan::plan_bytes(n_phases)) return DFL_ERR_WORKSPACE;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  int max_m = 0, flags_or = 0;
  for (int p = 0; p < n_phases; ++p) {
    const dfl_qmm_phase& q = phases[p];
    const bool grouped = (q.flags & kPhaseGrouped) != 0;
    if (q.M < 1 || q.M > (grouped ? kRouteMaxRows : kMaxRows) || q.K < 64 || q.K % 64 != 0 || q.N < 1 ||
        q.N > (1 << 24))
      return DFL_ERR_BAD_SHAPE;
    if ((q.flags & ~(kPhaseSilu | kPhaseSubnormal | kPhaseGrouped | kPhaseScatter)) != 0)
      return DFL_ERR_BAD_SHAPE;
    if ((q.flags & kPhaseScatter) && !grouped) return DFL_ERR_BAD_SHAPE;
    if (grouped) {
      // experts stacked whole tiles apart; at most kRouteMaxProblems problems
      // of at most problem_rows rows each, found in the sorted route table
      if (q.N % BN != 0 || q.experts < 1 || q.problem_rows < 1 || q.problem_rows > kMaxGroupedRows)
        return DFL_ERR_BAD_SHAPE;
      if (!q.route) return DFL_ERR_NULL_POINTER;
      if (!host::aligned(q.route, 4)) return DFL_ERR_MISALIGNED;
      const long long units = (long long)kRouteMaxProblems * (q.N / BN) * ((q.K + UNIT_K - 1) / UNIT_K);
      if (units > (1LL << 31) / (kMaxGrid + 1)) return DFL_ERR_BAD_SHAPE;
    }
    const bool silu = (q.flags & kPhaseSilu) != 0;
    if (silu && q.N % 32 != 0) return DFL_ERR_BAD_SHAPE;
    if (q.ldx < q.K || q.ldy < (silu ? q.N / 2 : q.N)) return DFL_ERR_BAD_SHAPE;
    if (q.dep < -1 || q.dep >= p) return DFL_ERR_BAD_SHAPE;
    if (!q.x || !q.y || !q.w_tiled) return DFL_ERR_NULL_POINTER;
    if (!host::aligned(q.x, 16) || q.ldx % 8 != 0 || !host::aligned(q.y, 2) ||
        !host::aligned(q.w_tiled, 16))
      return DFL_ERR_MISALIGNED;
    const long long tiles = (q.N + BN - 1) / BN, ku = (q.K + UNIT_K - 1) / UNIT_K;
    if (tiles * ku > (1LL << 31) / (kMaxGrid + 1)) return DFL_ERR_BAD_SHAPE;
    const int rows = grouped ? q.problem_rows : q.M;   // rows one token tile holds
    max_m = rows > max_m ? rows : max_m;
    flags_or |= q.flags;
  }
  const int mt = max_m <= 16 ? 16 : max_m <= 32 ? 32 : max_m <= 64 ? 64 : 128;
  if ((flags_or & kPhaseGrouped) && mt > kMaxGroupedRows) return DFL_ERR_BAD_SHAPE;
  // a grouped phase whose dep is a grouped phase over the same route table
  // waits per problem: the dep counts its stored tiles per problem in a
  // counter slot (at most kMaxProblemSlots; later pairs wait for the whole
  // phase as other dependencies do)
  std::vector<int> sig_slot(n_phases, 0), wait_slot(n_phases, 0);
  int slots = 0;
  for (int p = 0; p < n_phases; ++p) {
    const dfl_qmm_phase& q = phases[p];
    if (!(q.flags & kPhaseGrouped) || q.dep < 0) continue;
    const dfl_qmm_phase& d = phases[q.dep];
    if (!(d.flags & kPhaseGrouped) || d.route != q.route) continue;
    if (!sig_slot[q.dep] && slots < kMaxProblemSlots) sig_slot[q.dep] = ++slots;
    wait_slot[p] = sig_slot[q.dep];
  }
  uint8_t* out = static_cast<uint8_t*>(plan_host);
  Header h;
  std::memset(&h, 0, sizeof(h));
  h.magic = kPlanMagic;
  h.version = kPlanVersion;
  h.n_phases = n_phases;
  h.mt = mt;
  h.grid = sms < kMaxGrid ? sms : kMaxGrid;
  h.flags_or = flags_or;
  h.test_skip_partial_cta = -1;
  h.prob_slots = slots;
  h.wait_limit_ns = kWaitLimitNs;
  std::memcpy(out, &h, sizeof(h));
  for (int p = 0; p < n_phases; ++p) {
    const dfl_qmm_phase& q = phases[p];
    Phase ph;
    std::memset(&ph, 0, sizeof(ph));
    st = host::make_tmap_2d(&ph.tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q.x, uint64_t(q.K),
                            uint64_t(q.M), uint64_t(q.ldx) * 2, GS, mt, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DFL_OK) return st;
    ph.w = static_cast<const uint8_t*>(q.w_tiled);
    ph.y = static_cast<uint16_t*>(q.y);
    ph.M = q.M;
    ph.K = q.K;
    ph.N = q.N;
    ph.ldy = q.ldy;
    ph.n_tiles = (q.N + BN - 1) / BN;
    ph.ku = (q.K + UNIT_K - 1) / UNIT_K;
    ph.total = (q.flags & kPhaseGrouped) ? 0 : ph.n_tiles * ph.ku;   // grouped: from the route table
    const int n_out = (q.flags & kPhaseSilu) ? q.N / 2 : q.N;
    const bool vec = host::aligned(q.y, 16) && q.ldy % 8 == 0 && n_out % 8 == 0;
    ph.flags = q.flags | (sig_slot[p] << kSignalShift) | (wait_slot[p] << kWaitShift) | (vec ? kVecStore : 0);
    ph.dep = q.dep;
    ph.route = (q.flags & kPhaseGrouped) ? q.route : nullptr;
    ph.experts = (q.flags & kPhaseGrouped) ? q.experts : 0;
    std::memcpy(out + kHeaderBytes + size_t(p) * sizeof(Phase), &ph, sizeof(Phase));
  }
  return DFL_OK;
}

extern "C" size_t dfl_qmm_plan_workspace_bytes(const void* plan_host, int* status) {
  int dummy;
  int* st = status ? status : &dummy;
  dfl::plan::Header h;
  *st = dfl::plan::check_header(plan_host, &h);
  if (*st != DFL_OK) return 0;
  return dfl::plan::workspace_bytes(h.mt, h.grid);
}

extern "C" int dfl_qmm_plan_run(const void* plan_host, const void* plan_dev, void* workspace,
                                size_t workspace_bytes, void* stream) {
  using namespace dfl;
  plan::Header h;
  int st = plan::check_header(plan_host, &h);
  if (st != DFL_OK) return st;
  if (!plan_dev || !workspace) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(plan_dev, 64) || !host::aligned(workspace, 16)) return DFL_ERR_MISALIGNED;
  if (workspace_bytes < plan::workspace_bytes(h.mt, h.grid)) return DFL_ERR_WORKSPACE;
  int dev, sms;
  st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  if (h.grid > sms) return DFL_ERR_UNSUPPORTED;   // encoded for a larger device
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (h.mt) {
    case 16:
      return (h.flags_or & plan::kPhaseGrouped) ? plan::launch<16, true>(h, plan_dev, workspace, dev, s)
                                                : plan::launch<16, false>(h, plan_dev, workspace, dev, s);
    case 32:
      return (h.flags_or & plan::kPhaseGrouped) ? plan::launch<32, true>(h, plan_dev, workspace, dev, s)
                                                : plan::launch<32, false>(h, plan_dev, workspace, dev, s);
    case 64: return plan::launch<64, false>(h, plan_dev, workspace, dev, s);
    default: return plan::launch<128, false>(h, plan_dev, workspace, dev, s);
  }
}

extern "C" int dfl_qmm_plan_set_test_fault(void* plan_host, int skip_partial_cta,
                                           uint64_t wait_limit_ns) {
  dfl::plan::Header h;
  const int st = dfl::plan::check_header(plan_host, &h);
  if (st != DFL_OK) return st;
  if (skip_partial_cta < -1 || skip_partial_cta >= h.grid) return DFL_ERR_BAD_SHAPE;
  if (wait_limit_ns < 1000000ull || wait_limit_ns > dfl::kWaitLimitNs) return DFL_ERR_BAD_SHAPE;
  h.test_skip_partial_cta = skip_partial_cta;
  h.wait_limit_ns = wait_limit_ns;
  std::memcpy(plan_host, &h, sizeof(h));
  return DFL_OK;
}

extern "C" int dfl_qmm_plan_last_timeout(const void* workspace_host_words, int* role, int* phase,
                                         int* cta) {
  if (!workspace_host_words || !role || !phase || !cta) return DFL_ERR_NULL_POINTER;
  const int* w = static_cast<const int*>(workspace_host_words);
  const int where = w[dfl::plan::kWordWhere];
  *role = where >> 24;
  *phase = where & 0xFFFFFF;
  *cta = w[dfl::plan::kWordWhereCta];
  return DFL_OK;
}
