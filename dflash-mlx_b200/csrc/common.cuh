// Shared device helpers for the dflash-b200 kernels (sm_100a only).
//
// Thin inline-PTX wrappers for the Blackwell primitives the kernels use:
// mbarriers, TMA tiled loads (never with cluster multicast: these kernels
// run on every GPU of a multi-GPU job), tcgen05 TMEM allocation, loads,
// stores and MMAs, plus a bounded mbarrier wait that reports a time-out
// through a device error word instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "dflash-b200 kernels target sm_100a only"
#endif

namespace dfl {

// Error word written by kernels (time-outs, bad launch geometry).  Host code
// reads and clears it through dfl_get_device_error().  The library is one
// translation unit, so this header is included exactly once.
__device__ int g_device_error = 0;

enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,
  kDevBadGeometry = 2,
  kDevBadInput = 3,  // an index argument outside its documented range
};

// Upper bound on any single mbarrier wait.  A healthy wait finishes in
// microseconds; one second means the pipeline is broken.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Test for completion of the phase with the given parity.  A waiting thread
// is suspended (it issues nothing) until the phase completes or the hint of
// 10 ms runs out; without the hint waiting warps poll and take issue slots
// from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(10000000u)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// kWaitLimitNs, records kDevWaitTimeout and returns false; callers then
// leave their loops so the CTA can tear down (free TMEM) and exit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicExch(&g_device_error, kDevWaitTimeout);
      return false;
    }
  }
}

// Same, for kernels whose threads also meet at named barriers: leaving a
// loop early there could strand a barrier, so instead a time-out sets a
// CTA-wide abort word and every later wait returns false at once.  Threads
// keep walking the same control flow (skipping the issue of MMAs and copies)
// and the CTA reaches its teardown.
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity,
                                                    volatile int* abort_word) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort_word) return false;
  unsigned long long t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_word) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicExch(&g_device_error, kDevWaitTimeout);
      *abort_word = 1;
      return false;
    }
  }
}

// ------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while
// the previous kernel in the stream is still running.  griddep_wait() blocks
// until that kernel has completed and its memory is visible; everything that
// reads the previous kernel's outputs (or writes what it may still read) must
// come after it.  griddep_launch_dependents() lets the next such kernel start
// early.  Both are no-ops for a normal launch.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- cp.async
// 16-byte global -> shared copy through L2; src_bytes < 16 zero-fills the
// rest (0 reads nothing).
__device__ __forceinline__ void cp_async_16(uint32_t dst_smem, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst_smem), "l"(src),
               "r"(src_bytes)
               : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completing bytes on
// an mbarrier.  Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst_smem), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's earlier generic-proxy observations of global memory
// before its later async-proxy (bulk copy / TMA) reads of it.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// bf16 / fp16 bits of silu(g) * u computed in fp32 from the bits of g and u
// (the one definition every SiLU*up in this library uses).
template <bool F16>
__device__ __forceinline__ uint16_t silu_mul_bits(uint16_t gb, uint16_t ub) {
  float g, u;
  if constexpr (F16) {
    g = __half2float(__ushort_as_half(gb));
    u = __half2float(__ushort_as_half(ub));
  } else {
    g = __bfloat162float(__ushort_as_bfloat16(gb));
    u = __bfloat162float(__ushort_as_bfloat16(ub));
  }
  const float s = g / (1.0f + expf(-g));
  if constexpr (F16)
    return __half_as_ushort(__float2half_rn(s * u));
  else
    return __bfloat16_as_ushort(__float2bfloat16_rn(s * u));
}

// Warp sums of four values per lane (rows 0..3 of a warp, each spread over
// all 32 lanes) with 6 shuffles instead of 4 x 5: after the first two levels
// every lane carries one row; the result is the full sum of row
// ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1), held by the 8 lanes of that row.
__device__ __forceinline__ int row_of_lane4(int lane) { return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1); }

__device__ __forceinline__ float warp_reduce_rows4(const float (&v)[4], int lane) {
  const bool hi16 = (lane & 16) != 0;
  float a = hi16 ? v[2] : v[0];
  float b = hi16 ? v[3] : v[1];
  a += __shfl_xor_sync(0xffffffffu, hi16 ? v[0] : v[2], 16);
  b += __shfl_xor_sync(0xffffffffu, hi16 ? v[1] : v[3], 16);
  const bool hi8 = (lane & 8) != 0;
  float k = hi8 ? b : a;
  k += __shfl_xor_sync(0xffffffffu, hi8 ? a : b, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 1);
  return k;
}

// n consecutive floats of shared memory into registers, 16 bytes at a time
// when n % 4 == 0 (the address must then be 16-byte aligned).
template <int N>
__device__ __forceinline__ void lds_vec(const float* src, float (&r)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      r[i] = v.x; r[i + 1] = v.y; r[i + 2] = v.z; r[i + 3] = v.w;
    }
  } else if constexpr (N % 2 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 v = *reinterpret_cast<const float2*>(src + i);
      r[i] = v.x; r[i + 1] = v.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = src[i];
  }
}

// Relaxed (gpu scope, L2-coherent) 32-bit global load / store.  Each aligned
// 32-bit access is single-copy atomic, so a word that carries its own
// validity bit can be polled without a separate flag.
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_u32(uint32_t* addr, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

// Arrive at named barrier `id` of `count` threads without waiting for it.
// Like every bar.* form here it is an aligned barrier (each warp must reach
// it converged), so the calling warp is reconverged first: its lanes may
// come from different iterations of their own bounded waits.
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  __syncwarp();
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Release-add on a global counter (no return value): writes this thread
// observed before it (including other threads' writes ordered by a barrier)
// are visible to whoever acquires the new value.
__device__ __forceinline__ void red_release_add(int* addr, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire(const int* addr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Spin until *addr >= target (acquire).  Gives up like mbar_wait_abortable:
// after kWaitLimitNs, or at once when the CTA abort word is set.
__device__ __forceinline__ bool spin_acquire_geq(const int* addr, int target,
                                                 volatile int* abort_word) {
  if (ld_acquire(addr) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    __nanosleep(64);
    if (ld_acquire(addr) >= target) return true;
    if (*abort_word) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicExch(&g_device_error, kDevWaitTimeout);
      *abort_word = 1;
      return false;
    }
  }
}

// Close the current cp.async group / wait until at most N of this thread's
// most recent groups are still in flight.
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Wait until all of this thread's prior cp.async copies have landed.
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Arrive on an mbarrier once all of this thread's prior cp.async copies have
// landed; the arrival is counted in the barrier's expected count.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completion on an mbarrier.
// The innermost coordinate x times the element size is a multiple of 16
// bytes at every call site (checked on the host for each tensor map).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled bulk tensor load (x innermost); same alignment rule on x.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on an mbarrier when every tcgen05 op issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (bf16 operands, fp32 accumulate).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, shape M x N.
// Instruction descriptor for kind::f16 with fp32 accumulation and A, B both
// fp16 (f16 = true) or both bf16.
__host__ __device__ constexpr uint32_t make_idesc_16(int m, int n, bool f16) {
  return (1u << 4)                                  // D format f32
         | ((f16 ? 0u : 1u) << 7)                   // A format f16 / bf16
         | ((f16 ? 0u : 1u) << 10)                  // B format f16 / bf16
         | (uint32_t(n >> 3) << 17)                 // N / 8
         | (uint32_t(m >> 4) << 24);                // M / 16
}

__host__ __device__ constexpr uint32_t make_idesc_bf16(int m, int n) {
  return (1u << 4)                               // D format f32
         | (1u << 7)                             // A format bf16
         | (1u << 10)                            // B format bf16
         | (uint32_t(n >> 3) << 17)              // N / 8
         | (uint32_t(m >> 4) << 24);             // M / 16
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);        // start address
  d |= uint64_t(1u) << 16;                          // leading byte offset (unused for SW128 K-major)
  d |= uint64_t(1024u >> 4) << 32;                  // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1u) << 46;                          // descriptor version (sm100)
  d |= uint64_t(2u) << 61;                          // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 columns of 32-bit TMEM store (one lane per thread).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 columns of 32-bit TMEM load.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Named barrier over a subset of whole warps (aligned: reconverge first).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  __syncwarp();
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also returns the AND of `pred` over all participants
// (whole warps; aligned: reconverge first).
__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t nthreads, bool pred) {
  __syncwarp();
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %3, 0;\n\t"
      "bar.red.and.pred p, %1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(nthreads), "r"(pred ? 1u : 0u)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (TMA stores, tcgen05.mma operand fetches).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Warp-wide forms: every lane of the warp executes the call (so the operands
// stay warp-uniform) and one elected lane issues the instruction.
__device__ __forceinline__ void mma_bf16_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t elect_lane0() { return (threadIdx.x & 31u) == 0u; }

}  // namespace dfl
