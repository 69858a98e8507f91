// GatedDeltaNet tape-replay rollback (sm_100a).
//
// Replaces tape_replay_kernel (dflash_mlx/kernels.py:822-868, Metal body
// :708-758; mx-op reference _tape_replay_ops :790-820).  For every
// (sequence b, value head hv) and every step t that is replayed:
//     S[dv, dk] <- S[dv, dk] * g_t          (g_t scalar per head, or per dk)
//     S[dv, dk] <- S[dv, dk] + delta_t[dv] * k_t[dk]
// with k head hk = hv / (Hv / Hk) (kernels.py:712).  Step t of sequence b is
// replayed when t < steps[b] and mask[b, t] (either may be absent).  The two
// updates are separately rounded fp32 operations, exactly as the mx-op
// reference orders them, so results match it bit for bit.
//
// Layout: state [B, Hv, Dv, Dk] fp32, tape [B, T, Hv, Dv] fp32,
// k [B, T, Hk, Dk] (bf16 or fp32), g [B, T, Hv] or [B, T, Hv, Dk] fp32.
//
// One CTA per (b, hv) head, 256 threads.  The head's state (Dv x Dk fp32,
// 64 KB at 128 x 128) is read once with 16-byte coalesced loads into
// registers, all replayed steps are applied there (the step's k, delta and
// g sit in shared memory), and it is written back once.  A head with no step
// to replay is not touched when updating in place.  The kernel is HBM-bound:
// per replayed head 2 * Dv * Dk * 4 bytes of state plus a * (Dv + Hk/Hv-share
// of Dk) of tape.
#include "common.cuh"
#include "host_common.cuh"

namespace dfl {
namespace gdn {

constexpr int THREADS = 256;
constexpr int MAX_CHUNKS = 16;  // float4 state chunks per thread (Dv * Dk <= 16384)
constexpr int MAX_STEPS = 64;
// Largest staging area: MAX_STEPS * (Dv + 2 * Dk) floats with Dv * Dk <= 16384.
// (+16 bytes: the g region is padded to whole float4s)
constexpr int kMaxSmem = (MAX_STEPS * (512 + 2 * 32) * 4 > MAX_STEPS * (64 + 2 * 256) * 4
                              ? MAX_STEPS * (512 + 2 * 32) * 4
                              : MAX_STEPS * (64 + 2 * 256) * 4) + 16;

struct ReplayParams {
  const float* tape;
  const void* k;
  const float* g;
  const int32_t* steps;   // [B] or null (= T)
  const uint8_t* mask;    // [B, T] or null (= all)
  const float* state_in;
  float* state_out;
  int B, T, Hv, Hk, Dv, Dk;
  int g_vec;
  int vec;                // tape, k, g 16-byte aligned and Dv % 4 == 0: stage by cp.async
  int parts;              // CTAs per head (row slices of Dv / parts rows)
};

// Four consecutive k values from shared memory as floats (bf16 -> fp32 is exact).
template <typename KT>
__device__ __forceinline__ float4 load_k4(const KT* p);
template <>
__device__ __forceinline__ float4 load_k4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load_k4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
}

// Copy `rows` rows of `row_bytes` (a multiple of 16) from global rows
// `stride_bytes` apart into consecutive shared memory, 16 bytes per
// cp.async; every thread of the CTA takes a share.
__device__ __forceinline__ void stage_rows(uint8_t* dst, const uint8_t* src, int rows,
                                           int row_bytes, size_t stride_bytes, int tid) {
  const int per_row = row_bytes / 16;
  for (int i = tid; i < rows * per_row; i += THREADS) {
    const int r = i / per_row, c = i - r * per_row;
    cp_async_16(smem_u32(dst + (size_t)r * row_bytes + c * 16), src + r * stride_bytes + c * 16, 16);
  }
}

// NCH: float4 state chunks per thread (16: a whole head of up to 16384
// elements per CTA; 8: heads of more than 8192 elements split by rows over
// `parts` CTAs with half the registers, three CTAs per SM: 64 sequences x
// 48 layers x 48 heads of 128 x 128 in 5.10 ms instead of 5.44; four per SM
// spilled and was slower).
template <typename KT, int DK, int NCH>
__global__ void __launch_bounds__(THREADS, NCH <= 8 ? 3 : 1)
    tape_replay_kernel(const ReplayParams p) {
  extern __shared__ float sh[];
  const int head = blockIdx.x / p.parts;          // b * Hv + hv
  const int part = blockIdx.x - head * p.parts;
  const int rows = p.Dv / p.parts;                // value rows of this CTA
  const int r0 = part * rows;
  const int b = head / p.Hv;
  const int hv = head - b * p.Hv;
  const int hk = hv / (p.Hv / p.Hk);
  const int tid = threadIdx.x;

  int nsteps = p.steps ? p.steps[b] : p.T;
  nsteps = nsteps < 0 ? 0 : (nsteps > p.T ? p.T : nsteps);

  // Which of the first nsteps steps are replayed (mask), as a bit set.
  uint64_t active = 0;
  for (int t = 0; t < nsteps; ++t)
    if (!p.mask || p.mask[(size_t)b * p.T + t]) active |= (uint64_t(1) << t);

  const int dv_dk = rows * DK;
  const size_t sbase = (size_t)head * p.Dv * DK + (size_t)r0 * DK;
  const float4* src = reinterpret_cast<const float4*>(p.state_in + sbase);
  float4* dst = reinterpret_cast<float4*>(p.state_out + sbase);
  const int n4 = dv_dk / 4;

  if (active == 0) {
    if (p.state_in != p.state_out)
      for (int i = tid; i < n4; i += THREADS) dst[i] = src[i];
    return;
  }

  // The head's state first (16-byte loads into registers), so that it and the
  // staging copies below are all in flight together.  Thread tid owns float4
  // chunks f = j * THREADS + tid: row dv = 4f / DK, columns dk0..dk0+3 with
  // dk0 = 4f % DK = (4 * tid) % DK (DK divides 1024).
  float4 st[NCH];
  const int nchunk = (n4 + THREADS - 1) / THREADS;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int f = j * THREADS + tid;
    if (j < nchunk && f < n4) st[j] = __ldcs(src + f);
  }

  // Stage this head's replayed steps in shared memory: k [a][DK] (as stored),
  // g [a][DK] or [a], delta [a][Dv]; k and vector g first (16-byte rows).
  // Every region starts on a 16-byte boundary: k rows are DK * sizeof(KT) >= 64
  // bytes and the g region is padded to whole float4s.
  const int gw = p.g_vec ? DK : 1;
  KT* s_k = reinterpret_cast<KT*>(sh);
  float* s_g = reinterpret_cast<float*>(s_k + nsteps * DK);
  float* s_delta = s_g + ((nsteps * gw + 3) & ~3);
  const KT* kp = reinterpret_cast<const KT*>(p.k);
  // rows of step t: k row (b, t, hk), g row (b, t, hv), delta row (b, t, hv)
  const size_t k_row0 = ((size_t)b * p.T * p.Hk + hk) * DK;
  const size_t g_row0 = (size_t)b * p.T * p.Hv + hv;
  if (p.vec) {
    stage_rows(reinterpret_cast<uint8_t*>(s_k), reinterpret_cast<const uint8_t*>(kp + k_row0), nsteps,
               DK * int(sizeof(KT)), (size_t)p.Hk * DK * sizeof(KT), tid);
    if (p.g_vec)
      stage_rows(reinterpret_cast<uint8_t*>(s_g), reinterpret_cast<const uint8_t*>(p.g + g_row0 * DK),
                 nsteps, DK * 4, (size_t)p.Hv * DK * 4, tid);
    stage_rows(reinterpret_cast<uint8_t*>(s_delta),
               reinterpret_cast<const uint8_t*>(p.tape + g_row0 * p.Dv + r0), nsteps, rows * 4,
               (size_t)p.Hv * p.Dv * 4, tid);
  } else {
    for (int i = tid; i < nsteps * DK; i += THREADS) {
      const int t = i / DK, dk = i - t * DK;
      s_k[i] = kp[k_row0 + (size_t)t * p.Hk * DK + dk];
    }
    if (p.g_vec)
      for (int i = tid; i < nsteps * DK; i += THREADS) {
        const int t = i / DK, dk = i - t * DK;
        s_g[i] = p.g[(g_row0 + (size_t)t * p.Hv) * DK + dk];
      }
    for (int i = tid; i < nsteps * rows; i += THREADS) {
      const int t = i / rows, dv = i - t * rows;
      s_delta[i] = p.tape[(g_row0 + (size_t)t * p.Hv) * p.Dv + r0 + dv];
    }
  }
  if (!p.g_vec)
    for (int t = tid; t < nsteps; t += THREADS) s_g[t] = p.g[g_row0 + (size_t)t * p.Hv];
  cp_async_wait_all();
  __syncthreads();

  const int dk0 = (4 * tid) % DK;
  for (int t = 0; t < nsteps; ++t) {
    if (!((active >> t) & 1)) continue;
    const float4 kv = load_k4<KT>(s_k + t * DK + dk0);
    float4 gv;
    if (p.g_vec) {
      gv = *reinterpret_cast<const float4*>(s_g + t * DK + dk0);
    } else {
      const float g0 = s_g[t];
      gv = make_float4(g0, g0, g0, g0);
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int f = j * THREADS + tid;
      if (j < nchunk && f < n4) {
        const int dv = (4 * f) / DK;
        const float d = s_delta[t * rows + dv];
        float4 s = st[j];
        s.x = __fadd_rn(__fmul_rn(s.x, gv.x), __fmul_rn(d, kv.x));
        s.y = __fadd_rn(__fmul_rn(s.y, gv.y), __fmul_rn(d, kv.y));
        s.z = __fadd_rn(__fmul_rn(s.z, gv.z), __fmul_rn(d, kv.z));
        s.w = __fadd_rn(__fmul_rn(s.w, gv.w), __fmul_rn(d, kv.w));
        st[j] = s;
      }
    }
  }

#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int f = j * THREADS + tid;
    if (j < nchunk && f < n4) __stcs(dst + f, st[j]);
  }
}

template <typename KT, int NCH>
int launch_replay(const ReplayParams& p, cudaStream_t stream) {
  const int gw = p.g_vec ? p.Dk : 1;
  const size_t smem = size_t(p.T) * (p.Dv / p.parts + p.Dk + gw) * sizeof(float) + 16;
  const int grid = p.B * p.Hv * p.parts;
  switch (p.Dk) {
#define DFL_CASE(D)                                                                        \
  case D: {                                                                                \
    static std::atomic<uint64_t> done{0};                                                  \
    int dev = 0;                                                                           \
    if (cudaGetDevice(&dev) != cudaSuccess) return DFL_ERR_CUDA;                           \
    int st = host::ensure_smem(tape_replay_kernel<KT, D, NCH>, kMaxSmem, dev, done);        \
    if (st != DFL_OK) return st;                                                           \
    tape_replay_kernel<KT, D, NCH><<<grid, THREADS, smem, stream>>>(p);                    \
    break;                                                                                 \
  }
    DFL_CASE(32)
    DFL_CASE(64)
    DFL_CASE(128)
    DFL_CASE(256)
#undef DFL_CASE
    default:
      return DFL_ERR_BAD_SHAPE;
  }
  return host::launch_status();
}

}  // namespace gdn
}  // namespace dfl

extern "C" int dfl_gdn_tape_replay(const float* tape, const void* k, int k_is_bf16,
                                   const float* g, int g_vectorized, const int32_t* steps,
                                   const uint8_t* mask, const float* state_in, float* state_out,
                                   int B, int T, int Hv, int Hk, int Dv, int Dk, void* stream) {
  using namespace dfl;
  if (B < 0 || T < 0 || Hv < 1 || Hk < 1 || Dv < 1) return DFL_ERR_BAD_SHAPE;
  if (Hv % Hk != 0) return DFL_ERR_BAD_SHAPE;
  if (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256) return DFL_ERR_BAD_SHAPE;
  if ((long long)Dv * Dk > (long long)gdn::MAX_CHUNKS * gdn::THREADS * 4) return DFL_ERR_BAD_SHAPE;
  if (T > gdn::MAX_STEPS) return DFL_ERR_BAD_SHAPE;
  if (B == 0) return DFL_OK;
  if (!state_in || !state_out) return DFL_ERR_NULL_POINTER;
  if (T > 0 && (!tape || !k || !g)) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(state_in, 16) || !host::aligned(state_out, 16)) return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  gdn::ReplayParams p;
  p.tape = tape;
  p.k = k;
  p.g = g;
  p.steps = steps;
  p.mask = mask;
  p.state_in = state_in;
  p.state_out = state_out;
  p.B = B;
  p.T = T;
  p.Hv = Hv;
  p.Hk = Hk;
  p.Dv = Dv;
  p.Dk = Dk;
  p.g_vec = g_vectorized ? 1 : 0;
  p.vec = (Dv % 4 == 0 && host::aligned(tape, 16) && host::aligned(k, 16) && host::aligned(g, 16))
              ? 1 : 0;
  // heads of more than 8192 state elements: two CTAs of Dv / 2 rows each
  // (when the half keeps 16-byte rows of the tape: Dv / 2 % 4 == 0)
  const bool split = (long long)Dv * Dk > 8 * gdn::THREADS * 4 && Dv % 8 == 0;
  p.parts = split ? 2 : 1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (split)
    return k_is_bf16 ? gdn::launch_replay<__nv_bfloat16, 8>(p, s) : gdn::launch_replay<float, 8>(p, s);
  return k_is_bf16 ? gdn::launch_replay<__nv_bfloat16, 16>(p, s) : gdn::launch_replay<float, 16>(p, s);
}
