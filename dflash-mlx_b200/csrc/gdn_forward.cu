// GatedDeltaNet verify forward that records the innovation tape (sm_100a).
//
// Replaces gated_delta_kernel_with_tape (dflash_mlx/kernels.py:169-219, Metal
// body :28-101; mx-op reference _gated_delta_ops_with_tape :125-167).  For
// every sequence b, value head hv (k/q head hk = hv / (Hv / Hk)) and step t
// with mask[b, t] (mask absent: all steps):
//     S'      = S * g_t                    (g_t scalar per head, or per dk)
//     kv[dv]  = sum_dk S'[dv, dk] * k_t[dk]
//     delta   = (v_t[dv] - kv[dv]) * beta_t
//     S       = S' + k_t[dk] * delta[dv]
//     y_t[dv] = sum_dk S[dv, dk] * q_t[dk]          (bf16 out)
//     tape_t[dv] = delta[dv]                         (fp32)
// A masked-out step leaves S unchanged and writes tape = 0, y = 0.  The two
// state updates are separately rounded fp32 operations in the mx-op
// reference's order -- the same ones tape_replay_kernel applies -- so
// replaying this kernel's tape over the first a steps reproduces its state
// after a steps exactly.
//
// Layout: q, k [B, T, Hk, Dk] bf16; v [B, T, Hv, Dv] bf16; g [B, T, Hv] or
// [B, T, Hv, Dk] fp32; beta [B, T, Hv] fp32; state [B, Hv, Dv, Dk] fp32;
// y [B, T, Hv, Dv] bf16; tape [B, T, Hv, Dv] fp32.
//
// Mapping: a CTA of 8 warps owns 32 value rows of one head; a warp owns 4
// rows and lane l holds elements [l * Dk/32, (l+1) * Dk/32) of each, so the
// two dot products per row are Dk/32 FMAs per lane plus a butterfly (the four
// rows' reductions interleave).  The head's k, q and the CTA's v, g, beta for
// all T steps are staged in shared memory first, so the sequential step loop
// touches no global memory.  The state is read once and written once: the
// kernel is HBM-bound at B x Hv x Dv x Dk x 8 bytes of state traffic.

namespace dfl {
namespace gdnf {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int ROWS_PER_WARP = 4;
constexpr int ROWS = WARPS * ROWS_PER_WARP;  // value rows per CTA
constexpr int MAX_STEPS = 64;

struct FwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* g;
  const float* beta;
  const uint8_t* mask;  // [B, T] or null
  const float* state_in;
  float* state_out;
  __nv_bfloat16* y;
  float* tape;
  int B, T, Hv, Hk, Dv, Dk;
  int g_vec;
};

__host__ __device__ constexpr size_t smem_bytes(int T, int Dk, int g_vec) {
  // k and q as float [T][Dk], g [T][Dk] or [T], beta [T], v [T][ROWS], mask [T]
  return size_t(T) * Dk * 4 * 2 + size_t(T) * (g_vec ? Dk : 1) * 4 + size_t(T) * 4 +
         size_t(T) * ROWS * 4 + size_t(T) * 4;
}

template <int NPL>
__device__ __forceinline__ void load_row(const float* src, float (&r)[NPL]) {
  if constexpr (NPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < NPL; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      r[i] = v.x; r[i + 1] = v.y; r[i + 2] = v.z; r[i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NPL; ++i) r[i] = src[i];
  }
}

template <int NPL>
__device__ __forceinline__ void store_row(float* dst, const float (&r)[NPL]) {
  if constexpr (NPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < NPL; i += 4)
      *reinterpret_cast<float4*>(dst + i) = make_float4(r[i], r[i + 1], r[i + 2], r[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < NPL; ++i) dst[i] = r[i];
  }
}

template <int DK>
__global__ void __launch_bounds__(THREADS) gdn_forward_tape_kernel(const FwdParams p) {
  constexpr int NPL = DK / 32;  // state elements of a row per lane
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int T = p.T;
  float* k_s = reinterpret_cast<float*>(smem_raw);          // [T][DK]
  float* q_s = k_s + T * DK;                                // [T][DK]
  float* g_s = q_s + T * DK;                                // [T][DK] or [T]
  float* b_s = g_s + T * (p.g_vec ? DK : 1);                // [T]
  float* v_s = b_s + T;                                     // [T][ROWS]
  int* m_s = reinterpret_cast<int*>(v_s + T * ROWS);        // [T]

  const int blocks_per_head = p.Dv / ROWS;
  const int n = blockIdx.x / blocks_per_head;  // b * Hv + hv
  const int row0 = (blockIdx.x - n * blocks_per_head) * ROWS;
  const int b = n / p.Hv;
  const int hv = n - b * p.Hv;
  const int hk = hv / (p.Hv / p.Hk);

  // ---- stage the head's per-step inputs
  for (int i = threadIdx.x; i < T * DK; i += THREADS) {
    const int t = i / DK, d = i - t * DK;
    const size_t kq = (((size_t)b * T + t) * p.Hk + hk) * DK + d;
    k_s[i] = __bfloat162float(p.k[kq]);
    q_s[i] = __bfloat162float(p.q[kq]);
    if (p.g_vec) g_s[i] = p.g[(((size_t)b * T + t) * p.Hv + hv) * DK + d];
  }
  for (int i = threadIdx.x; i < T * ROWS; i += THREADS) {
    const int t = i / ROWS, r = i - t * ROWS;
    v_s[i] = __bfloat162float(p.v[(((size_t)b * T + t) * p.Hv + hv) * p.Dv + row0 + r]);
  }
  for (int t = threadIdx.x; t < T; t += THREADS) {
    const size_t bt = ((size_t)b * T + t) * p.Hv + hv;
    if (!p.g_vec) g_s[t] = p.g[bt];
    b_s[t] = p.beta[bt];
    m_s[t] = p.mask ? (p.mask[(size_t)b * T + t] != 0) : 1;
  }

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c0 = lane * NPL;  // this lane's first dk
  float s[ROWS_PER_WARP][NPL];
  const size_t head_off = (size_t)n * p.Dv * DK;
#pragma unroll
  for (int j = 0; j < ROWS_PER_WARP; ++j)
    load_row<NPL>(p.state_in + head_off + (size_t)(row0 + warp * ROWS_PER_WARP + j) * DK + c0, s[j]);
  __syncthreads();

  static_assert(ROWS_PER_WARP == 4, "warp_reduce_rows4 reduces four rows");
  const int my_row = row_of_lane4(lane);  // the row whose sums this lane ends up with
  const bool writer = (lane & 7) == 0;    // lanes 0, 8, 16, 24 write rows 0..3
  for (int t = 0; t < T; ++t) {
    float kt[NPL], qt[NPL], gv[NPL];
    lds_vec<NPL>(k_s + t * DK + c0, kt);
    lds_vec<NPL>(q_s + t * DK + c0, qt);
    if (p.g_vec) {
      lds_vec<NPL>(g_s + t * DK + c0, gv);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) gv[i] = g_s[t];
    }
    const size_t out_off = (((size_t)b * T + t) * p.Hv + hv) * p.Dv + row0 + warp * ROWS_PER_WARP;
    if (!m_s[t]) {
      if (writer) {
        p.tape[out_off + my_row] = 0.f;
        p.y[out_off + my_row] = __float2bfloat16_rn(0.f);
      }
      continue;
    }
    float kv[ROWS_PER_WARP];
#pragma unroll
    for (int j = 0; j < ROWS_PER_WARP; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        s[j][i] = __fmul_rn(s[j][i], gv[i]);
        acc = __fmaf_rn(s[j][i], kt[i], acc);
      }
      kv[j] = acc;
    }
    // the row's delta is formed by the lanes holding its sum, then broadcast
    const float kv_row = warp_reduce_rows4(kv, lane);
    const float d_row =
        __fmul_rn(__fsub_rn(v_s[t * ROWS + warp * ROWS_PER_WARP + my_row], kv_row), b_s[t]);
    float out[ROWS_PER_WARP];
#pragma unroll
    for (int j = 0; j < ROWS_PER_WARP; ++j) {
      const float dj = __shfl_sync(0xffffffffu, d_row, 8 * (j & 1) + 16 * (j >> 1));
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        s[j][i] = __fadd_rn(s[j][i], __fmul_rn(kt[i], dj));
        acc = __fmaf_rn(s[j][i], qt[i], acc);
      }
      out[j] = acc;
    }
    const float out_row = warp_reduce_rows4(out, lane);
    if (writer) {
      p.tape[out_off + my_row] = d_row;
      p.y[out_off + my_row] = __float2bfloat16_rn(out_row);
    }
  }

#pragma unroll
  for (int j = 0; j < ROWS_PER_WARP; ++j)
    store_row<NPL>(p.state_out + head_off + (size_t)(row0 + warp * ROWS_PER_WARP + j) * DK + c0, s[j]);
}

// Dk = 128 variant: a CTA of 128 threads owns 64 value rows of one head;
// four consecutive lanes share a pair of rows and lane quad q holds columns
// 16 i + 4 q + e (i < 8, e < 4) of both, so each step is 10 FP32 operations
// per shared-memory load or shuffle (k / q chunks are broadcast loads: the
// lanes of a row pair read 64 contiguous bytes), a dot product ends in two
// butterfly shuffles inside the four lanes (each lane gets the same sum),
// and state rows load and store as 64-byte pieces.  Same operations and
// update order as the general kernel (the tape replays exactly).  The
// kernel is bound by FP32 issue: 5 operations per state element and step
// (decay, two for the rank-1 update, two dot-product FMAs).
constexpr int K128_THREADS = 128;
constexpr int K128_ROWS = 64;

__host__ __device__ constexpr size_t smem_bytes_k128(int T, int g_vec) {
  return size_t(T) * 128 * 4 * 2 + size_t(T) * (g_vec ? 128 : 1) * 4 + size_t(T) * 4 +
         size_t(T) * K128_ROWS * 4 + size_t(T) * 4;
}

__device__ __forceinline__ float4 lds_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__global__ void __launch_bounds__(K128_THREADS, 4) gdn_forward_tape_k128(const FwdParams p) {
  constexpr int DK = 128;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int T = p.T;
  float* k_s = reinterpret_cast<float*>(smem_raw);          // [T][128]
  float* q_s = k_s + T * DK;                                // [T][128]
  float* g_s = q_s + T * DK;                                // [T][128] or [T]
  float* b_s = g_s + T * (p.g_vec ? DK : 1);                // [T]
  float* v_s = b_s + T;                                     // [T][64]
  int* m_s = reinterpret_cast<int*>(v_s + T * K128_ROWS);   // [T]

  const int blocks_per_head = p.Dv / K128_ROWS;
  const int n = blockIdx.x / blocks_per_head;  // b * Hv + hv
  const int row0 = (blockIdx.x - n * blocks_per_head) * K128_ROWS;
  const int b = n / p.Hv;
  const int hv = n - b * p.Hv;
  const int hk = hv / (p.Hv / p.Hk);

  for (int i = threadIdx.x; i < T * DK; i += K128_THREADS) {
    const int t = i / DK, d = i - t * DK;
    const size_t kq = (((size_t)b * T + t) * p.Hk + hk) * DK + d;
    k_s[i] = __bfloat162float(p.k[kq]);
    q_s[i] = __bfloat162float(p.q[kq]);
    if (p.g_vec) g_s[i] = p.g[(((size_t)b * T + t) * p.Hv + hv) * DK + d];
  }
  for (int i = threadIdx.x; i < T * K128_ROWS; i += K128_THREADS) {
    const int t = i / K128_ROWS, r = i - t * K128_ROWS;
    v_s[i] = __bfloat162float(p.v[(((size_t)b * T + t) * p.Hv + hv) * p.Dv + row0 + r]);
  }
  for (int t = threadIdx.x; t < T; t += K128_THREADS) {
    const size_t bt = ((size_t)b * T + t) * p.Hv + hv;
    if (!p.g_vec) g_s[t] = p.g[bt];
    b_s[t] = p.beta[bt];
    m_s[t] = p.mask ? (p.mask[(size_t)b * T + t] != 0) : 1;
  }

  const int quad = threadIdx.x & 3;
  const int pr = threadIdx.x >> 2;             // row pair
  const int ra = row0 + 2 * pr;                // rows ra, ra + 1
  const size_t head_off = (size_t)n * p.Dv * DK;
  const float* src0 = p.state_in + head_off + (size_t)ra * DK + 4 * quad;
  float s0[32], s1[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 a = *reinterpret_cast<const float4*>(src0 + 16 * i);
    const float4 c = *reinterpret_cast<const float4*>(src0 + DK + 16 * i);
    s0[4 * i] = a.x; s0[4 * i + 1] = a.y; s0[4 * i + 2] = a.z; s0[4 * i + 3] = a.w;
    s1[4 * i] = c.x; s1[4 * i + 1] = c.y; s1[4 * i + 2] = c.z; s1[4 * i + 3] = c.w;
  }
  __syncthreads();

  for (int t = 0; t < T; ++t) {
    const size_t out_off = (((size_t)b * T + t) * p.Hv + hv) * p.Dv + ra;
    if (!m_s[t]) {
      if (quad == 0) {
        p.tape[out_off] = 0.f;
        p.tape[out_off + 1] = 0.f;
        p.y[out_off] = __float2bfloat16_rn(0.f);
        p.y[out_off + 1] = __float2bfloat16_rn(0.f);
      }
      continue;
    }
    const float* kt = k_s + t * DK + 4 * quad;
    const float* qt = q_s + t * DK + 4 * quad;
    const float* gt = g_s + (p.g_vec ? t * DK + 4 * quad : t);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 k4 = lds_f4(kt + 16 * i);
      float4 g4;
      if (p.g_vec) {
        g4 = lds_f4(gt + 16 * i);
      } else {
        g4.x = g4.y = g4.z = g4.w = *gt;
      }
      const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
      const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s0[4 * i + e] = __fmul_rn(s0[4 * i + e], gg[e]);
        s1[4 * i + e] = __fmul_rn(s1[4 * i + e], gg[e]);
        a0 = __fmaf_rn(s0[4 * i + e], kk[e], a0);
        a1 = __fmaf_rn(s1[4 * i + e], kk[e], a1);
      }
    }
    a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
    a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
    a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
    a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
    const float d0 = __fmul_rn(__fsub_rn(v_s[t * K128_ROWS + 2 * pr], a0), b_s[t]);
    const float d1 = __fmul_rn(__fsub_rn(v_s[t * K128_ROWS + 2 * pr + 1], a1), b_s[t]);
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 k4 = lds_f4(kt + 16 * i);
      const float4 q4 = lds_f4(qt + 16 * i);
      const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
      const float qq[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s0[4 * i + e] = __fadd_rn(s0[4 * i + e], __fmul_rn(kk[e], d0));
        s1[4 * i + e] = __fadd_rn(s1[4 * i + e], __fmul_rn(kk[e], d1));
        y0 = __fmaf_rn(s0[4 * i + e], qq[e], y0);
        y1 = __fmaf_rn(s1[4 * i + e], qq[e], y1);
      }
    }
    y0 = __fadd_rn(y0, __shfl_xor_sync(0xffffffffu, y0, 1));
    y1 = __fadd_rn(y1, __shfl_xor_sync(0xffffffffu, y1, 1));
    y0 = __fadd_rn(y0, __shfl_xor_sync(0xffffffffu, y0, 2));
    y1 = __fadd_rn(y1, __shfl_xor_sync(0xffffffffu, y1, 2));
    if (quad == 0) {
      p.tape[out_off] = d0;
      p.tape[out_off + 1] = d1;
      p.y[out_off] = __float2bfloat16_rn(y0);
      p.y[out_off + 1] = __float2bfloat16_rn(y1);
    }
  }

  float* dst0 = p.state_out + head_off + (size_t)ra * DK + 4 * quad;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    *reinterpret_cast<float4*>(dst0 + 16 * i) =
        make_float4(s0[4 * i], s0[4 * i + 1], s0[4 * i + 2], s0[4 * i + 3]);
    *reinterpret_cast<float4*>(dst0 + DK + 16 * i) =
        make_float4(s1[4 * i], s1[4 * i + 1], s1[4 * i + 2], s1[4 * i + 3]);
  }
}

inline int launch_forward_k128(const FwdParams& p, cudaStream_t stream) {
  static std::atomic<uint64_t> smem_done{0};
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  st = host::ensure_smem(gdn_forward_tape_k128, int(smem_bytes_k128(MAX_STEPS, 1)), dev, smem_done);
  if (st != DFL_OK) return st;
  const int grid = p.B * p.Hv * (p.Dv / K128_ROWS);
  gdn_forward_tape_k128<<<grid, K128_THREADS, smem_bytes_k128(p.T, p.g_vec), stream>>>(p);
  return host::launch_status();
}

template <int DK>
int launch_forward(const FwdParams& p, cudaStream_t stream) {
  if (DK == 128 && p.Dv % K128_ROWS == 0) return launch_forward_k128(p, stream);
  static std::atomic<uint64_t> smem_done{0};
  const size_t smem = smem_bytes(p.T, DK, p.g_vec);
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  st = host::ensure_smem(gdn_forward_tape_kernel<DK>, int(smem_bytes(MAX_STEPS, DK, 1)), dev,
                         smem_done);
  if (st != DFL_OK) return st;
  const int grid = p.B * p.Hv * (p.Dv / ROWS);
  gdn_forward_tape_kernel<DK><<<grid, THREADS, smem, stream>>>(p);
  return host::launch_status();
}

}  // namespace gdnf
}  // namespace dfl

extern "C" int dfl_gdn_forward_tape(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                    const float* g, int g_vectorized, const float* beta,
                                    const uint8_t* mask, const float* state_in, float* state_out,
                                    uint16_t* y, float* tape, int B, int T, int Hv, int Hk, int Dv,
                                    int Dk, void* stream) {
  using namespace dfl;
  if (B < 0 || T < 0 || Hv < 1 || Hk < 1 || Dv < 1 || Hv % Hk != 0) return DFL_ERR_BAD_SHAPE;
  if (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256) return DFL_ERR_BAD_SHAPE;
  if (Dv % gdnf::ROWS != 0 || T > gdnf::MAX_STEPS) return DFL_ERR_BAD_SHAPE;
  if (B == 0) return DFL_OK;
  if (!state_in || !state_out) return DFL_ERR_NULL_POINTER;
  if (T > 0 && (!q || !k || !v || !g || !beta || !y || !tape)) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(state_in, 16) || !host::aligned(state_out, 16)) return DFL_ERR_MISALIGNED;
  gdnf::FwdParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.g = g;
  p.beta = beta;
  p.mask = mask;
  p.state_in = state_in;
  p.state_out = state_out;
  p.y = reinterpret_cast<__nv_bfloat16*>(y);
  p.tape = tape;
  p.B = B;
  p.T = T;
  p.Hv = Hv;
  p.Hk = Hk;
  p.Dv = Dv;
  p.Dk = Dk;
  p.g_vec = g_vectorized ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (Dk) {
    case 32: return gdnf::launch_forward<32>(p, s);
    case 64: return gdnf::launch_forward<64>(p, s);
    case 128: return gdnf::launch_forward<128>(p, s);
    default: return gdnf::launch_forward<256>(p, s);
  }
}
