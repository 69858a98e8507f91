// DDTree verify kernels (sm_100a): the GatedDeltaNet recurrence over a token
// tree, and the tree-path depthwise causal conv1d in front of it.
//
// gdn_tree_kernel replaces gated_delta_tree_kernel and
// gated_delta_tree_tape_kernel (dflash_mlx/kernels.py:501-586; Metal bodies
// :222-420; mx-op references _gated_delta_tree_ops / _tree_tape_ops
// :421-498).  Tree node t (0 <= t < T, parents before children) starts from
// the state of node parent_ids[t], or from state_in when parent_ids[t] < 0,
// and applies one gated delta step:
//     S'      = S_parent * g_t                  (g_t per head, or per dk)
//     kv[dv]  = sum_dk S'[dv, dk] * k_t[dk]
//     delta   = (v_t[dv] - kv[dv]) * beta_t
//     S_t     = S' + k_t[dk] * delta[dv]
//     y_t[dv] = sum_dk S_t[dv, dk] * q_t[dk]
// Every node's state S_t goes to node_states [B, T, Hv, Dv, Dk] (fp32; the
// tree kernel's tree_states output, the tape variant's scratch), and with a
// tape pointer delta goes to tape [B, T, Hv, Dv] (fp32).  The two state
// updates are separately rounded fp32 operations in the reference's order,
// the ones tape_replay_kernel applies, so replaying the tape rows of a
// root-to-node path from state_in reproduces S_node exactly.  A parent id
// outside [-1, t) is a caller error: it is recorded in the device error word
// (kDevBadInput) and the node starts from state_in instead.
//
// Mapping (as gdn_forward.cu): a CTA of 8 warps owns 32 value rows of one
// head (rows >= Dv idle), a warp 4 rows, lane l the dk slice
// [l * Dk/32, (l+1) * Dk/32).  The head's k, q, g, beta, v and the parent
// list are staged in shared memory; a node's parent state is read back from
// node_states, which the same threads wrote for the parent.
//
// tree_conv1d_kernel replaces tree_depthwise_conv1d (kernels.py:647-688;
// Metal body :588-629; mx-op reference _tree_depthwise_conv1d_ops
// :631-644): out[b, t, c] = silu(sum_w x(slot_w) * weight[c, w] (+ bias[c]))
// with slot_w = path_indices[t, w] indexing the concatenation
// [prefix[b] (K-1 rows), qkv[b] (T rows)], fp32 accumulation in w order.
// A slot outside [0, K-1+T) is a caller error (kDevBadInput) and reads 0.

namespace dfl {
namespace gdntree {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int ROWS_PER_WARP = 4;
constexpr int ROWS = WARPS * ROWS_PER_WARP;
constexpr int MAX_NODES = 64;

struct TreeParams {
  const void* q;  // [B, T, Hk, Dk] (InT)
  const void* k;
  const void* v;  // [B, T, Hv, Dv] (InT)
  const float* g;
  const float* beta;
  const float* state_in;     // [B, Hv, Dv, Dk]
  const int* parent_ids;     // [T]
  void* y;                   // [B, T, Hv, Dv] (InT)
  float* node_states;        // [B, T, Hv, Dv, Dk]
  float* tape;               // [B, T, Hv, Dv] or null
  int B, T, Hv, Hk, Dv, Dk;
  int g_vec;
};

__host__ __device__ constexpr size_t tree_smem_bytes(int T, int Dk, int g_vec) {
  return size_t(T) * Dk * 4 * 2 + size_t(T) * (g_vec ? Dk : 1) * 4 + size_t(T) * 4 +
         size_t(T) * ROWS * 4 + size_t(T) * 4;
}

template <typename InT>
__device__ __forceinline__ float to_f(InT v) {
  if constexpr (std::is_same<InT, float>::value)
    return v;
  else
    return __bfloat162float(v);
}

template <typename InT>
__device__ __forceinline__ InT from_f(float v) {
  if constexpr (std::is_same<InT, float>::value)
    return v;
  else
    return __float2bfloat16_rn(v);
}

template <int NPL>
__device__ __forceinline__ void load_slice(const float* src, float (&r)[NPL]) {
#pragma unroll
  for (int i = 0; i < NPL; ++i) r[i] = src[i];
}

template <int NPL>
__device__ __forceinline__ void store_slice(float* dst, const float (&r)[NPL]) {
#pragma unroll
  for (int i = 0; i < NPL; ++i) dst[i] = r[i];
}

template <int DK, typename InT>
__global__ void __launch_bounds__(THREADS) gdn_tree_kernel(const TreeParams p) {
  constexpr int NPL = DK / 32;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int T = p.T;
  float* k_s = reinterpret_cast<float*>(smem_raw);  // [T][DK]
  float* q_s = k_s + T * DK;                        // [T][DK]
  float* g_s = q_s + T * DK;                        // [T][DK] or [T]
  float* b_s = g_s + T * (p.g_vec ? DK : 1);        // [T]
  float* v_s = b_s + T;                             // [T][ROWS]
  int* par_s = reinterpret_cast<int*>(v_s + T * ROWS);  // [T]
  const InT* q = static_cast<const InT*>(p.q);
  const InT* k = static_cast<const InT*>(p.k);
  const InT* v = static_cast<const InT*>(p.v);
  InT* y = static_cast<InT*>(p.y);

  const int blocks_per_head = (p.Dv + ROWS - 1) / ROWS;
  const int n = blockIdx.x / blocks_per_head;  // b * Hv + hv
  const int row0 = (blockIdx.x - n * blocks_per_head) * ROWS;
  const int b = n / p.Hv;
  const int hv = n - b * p.Hv;
  const int hk = hv / (p.Hv / p.Hk);

  for (int i = threadIdx.x; i < T * DK; i += THREADS) {
    const int t = i / DK, d = i - t * DK;
    const size_t kq = (((size_t)b * T + t) * p.Hk + hk) * DK + d;
    k_s[i] = to_f<InT>(k[kq]);
    q_s[i] = to_f<InT>(q[kq]);
    if (p.g_vec) g_s[i] = p.g[(((size_t)b * T + t) * p.Hv + hv) * DK + d];
  }
  for (int i = threadIdx.x; i < T * ROWS; i += THREADS) {
    const int t = i / ROWS, r = i - t * ROWS;
    v_s[i] = row0 + r < p.Dv ? to_f<InT>(v[(((size_t)b * T + t) * p.Hv + hv) * p.Dv + row0 + r]) : 0.f;
  }
  for (int t = threadIdx.x; t < T; t += THREADS) {
    const size_t bt = ((size_t)b * T + t) * p.Hv + hv;
    if (!p.g_vec) g_s[t] = p.g[bt];
    b_s[t] = p.beta[bt];
    int par = p.parent_ids[t];
    if (par < -1 || par >= t) {
      if (blockIdx.x == 0) atomicExch(&g_device_error, kDevBadInput);
      par = -1;
    }
    par_s[t] = par;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rw = row0 + warp * ROWS_PER_WARP;  // this warp's first value row
  if (rw >= p.Dv) return;                      // Dv % 4 == 0: whole warps idle
  const int c0 = lane * NPL;
  const size_t head_rows = (size_t)n * p.Dv;   // row index base of (b, hv) in state_in
  float s[ROWS_PER_WARP][NPL];

  for (int t = 0; t < T; ++t) {
    const int par = par_s[t];
    // node states are [B, T, Hv, Dv, Dk]: node (b, u) of head hv, row r
    auto node_row = [&](int u, int r) {
      return p.node_states + ((((size_t)b * T + u) * p.Hv + hv) * p.Dv + r) * DK + c0;
    };
#pragma unroll
    for (int j = 0; j < ROWS_PER_WARP; ++j)
      load_slice<NPL>(par < 0 ? p.state_in + (head_rows + rw + j) * DK + c0 : node_row(par, rw + j), s[j]);
    float kt[NPL], qt[NPL], gv[NPL];
    lds_vec<NPL>(k_s + t * DK + c0, kt);
    lds_vec<NPL>(q_s + t * DK + c0, qt);
    if (p.g_vec) {
      lds_vec<NPL>(g_s + t * DK + c0, gv);
    } else {
#pragma unroll
      for (int i = 0; i < NPL; ++i) gv[i] = g_s[t];
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
    // the lanes holding a row's sum form its delta; then it is broadcast
    const int my_row = row_of_lane4(lane);
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
#pragma unroll
    for (int j = 0; j < ROWS_PER_WARP; ++j) store_slice<NPL>(node_row(t, rw + j), s[j]);
    if ((lane & 7) == 0) {
      const size_t o = (((size_t)b * T + t) * p.Hv + hv) * p.Dv + rw + my_row;
      y[o] = from_f<InT>(out_row);
      if (p.tape) p.tape[o] = d_row;
    }
  }
}

template <int DK, typename InT>
int launch_tree(const TreeParams& p, cudaStream_t stream) {
  static std::atomic<uint64_t> smem_done{0};
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  st = host::ensure_smem(gdn_tree_kernel<DK, InT>, int(tree_smem_bytes(MAX_NODES, DK, 1)), dev,
                         smem_done);
  if (st != DFL_OK) return st;
  const int grid = p.B * p.Hv * ((p.Dv + ROWS - 1) / ROWS);
  gdn_tree_kernel<DK, InT><<<grid, THREADS, tree_smem_bytes(p.T, DK, p.g_vec), stream>>>(p);
  return host::launch_status();
}

template <typename InT>
__global__ void tree_conv1d_kernel(const InT* __restrict__ qkv, const InT* __restrict__ prefix,
                                   const float* __restrict__ weight, const float* __restrict__ bias,
                                   const int* __restrict__ path, InT* __restrict__ out, int B,
                                   int T, int C, int K) {
  const size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (i >= (size_t)B * T * C) return;
  const int c = int(i % C);
  const int t = int((i / C) % T);
  const int b = int(i / ((size_t)C * T));
  const int pre = K - 1;
  float acc = 0.f;
  for (int w = 0; w < K; ++w) {
    const int slot = path[t * K + w];
    float x = 0.f;
    if (slot >= 0 && slot < pre)
      x = to_f<InT>(prefix[((size_t)b * pre + slot) * C + c]);
    else if (slot >= pre && slot < pre + T)
      x = to_f<InT>(qkv[((size_t)b * T + (slot - pre)) * C + c]);
    else if (c == 0 && b == 0)
      atomicExch(&g_device_error, kDevBadInput);
    acc = __fmaf_rn(x, weight[(size_t)c * K + w], acc);
  }
  if (bias) acc = __fadd_rn(acc, bias[c]);
  out[i] = from_f<InT>(acc / (1.0f + expf(-acc)));
}

}  // namespace gdntree
}  // namespace dfl

extern "C" int dfl_gdn_tree_forward(const void* q, const void* k, const void* v, const float* g,
                                    int g_vectorized, const float* beta, const float* state_in,
                                    const int32_t* parent_ids, void* y, float* node_states,
                                    float* tape, int B, int T, int Hv, int Hk, int Dv, int Dk,
                                    int inputs_f32, void* stream) {
  using namespace dfl;
  if (B < 0 || T < 0 || Hv < 1 || Hk < 1 || Dv < 1 || Hv % Hk != 0) return DFL_ERR_BAD_SHAPE;
  if (Dk != 32 && Dk != 64 && Dk != 128 && Dk != 256) return DFL_ERR_BAD_SHAPE;
  if (Dv % gdntree::ROWS_PER_WARP != 0 || T > gdntree::MAX_NODES) return DFL_ERR_BAD_SHAPE;
  if (B == 0 || T == 0) return DFL_OK;
  if (!q || !k || !v || !g || !beta || !state_in || !parent_ids || !y || !node_states)
    return DFL_ERR_NULL_POINTER;
  gdntree::TreeParams p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.g = g;
  p.beta = beta;
  p.state_in = state_in;
  p.parent_ids = parent_ids;
  p.y = y;
  p.node_states = node_states;
  p.tape = tape;
  p.B = B;
  p.T = T;
  p.Hv = Hv;
  p.Hk = Hk;
  p.Dv = Dv;
  p.Dk = Dk;
  p.g_vec = g_vectorized ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (inputs_f32) {
    switch (Dk) {
      case 32: return gdntree::launch_tree<32, float>(p, s);
      case 64: return gdntree::launch_tree<64, float>(p, s);
      case 128: return gdntree::launch_tree<128, float>(p, s);
      default: return gdntree::launch_tree<256, float>(p, s);
    }
  }
  switch (Dk) {
    case 32: return gdntree::launch_tree<32, __nv_bfloat16>(p, s);
    case 64: return gdntree::launch_tree<64, __nv_bfloat16>(p, s);
    case 128: return gdntree::launch_tree<128, __nv_bfloat16>(p, s);
    default: return gdntree::launch_tree<256, __nv_bfloat16>(p, s);
  }
}

extern "C" int dfl_tree_depthwise_conv1d(const void* qkv, const void* prefix, const float* weight,
                                         const float* bias, const int32_t* path_indices, void* out,
                                         int B, int T, int C, int K, int inputs_f32,
                                         void* stream) {
  using namespace dfl;
  if (B < 0 || T < 0 || C < 1 || K < 1) return DFL_ERR_BAD_SHAPE;
  const size_t total = (size_t)B * T * C;
  if (total == 0) return DFL_OK;
  if (!qkv || !weight || !path_indices || !out || (K > 1 && !prefix)) return DFL_ERR_NULL_POINTER;
  const int threads = 256;
  const unsigned blocks = unsigned((total + threads - 1) / threads);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (inputs_f32)
    gdntree::tree_conv1d_kernel<float><<<blocks, threads, 0, s>>>(
        static_cast<const float*>(qkv), static_cast<const float*>(prefix), weight, bias,
        path_indices, static_cast<float*>(out), B, T, C, K);
  else
    gdntree::tree_conv1d_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(prefix), weight,
        bias, path_indices, static_cast<__nv_bfloat16*>(out), B, T, C, K);
  return host::launch_status();
}
