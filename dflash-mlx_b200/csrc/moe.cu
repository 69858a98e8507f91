// MoE verify helpers around the grouped int4 qmm (qmm_w4.cu):
//   * routing: top-k experts per token by router logit (ties to the lower
//     expert id), softmax over the k kept logits (equal to softmax over all
//     experts followed by renormalisation of the kept probabilities), and a
//     route table listing the active experts with their tokens;
//   * silu(gate) * up in fp32, rounded to bf16;
//   * the weighted combine y_t = sum_j w[t, j] * out[t*k + j] (+ shared expert).
// The expert block restated here is mlx-lm's SwitchGLU (third party, not in
// the reference tree), reached from dflash_mlx/engine/target_qwen_gdn.py:863-865.
#include "common.cuh"
#include "host_common.cuh"

namespace dfl {
namespace moe {

constexpr int MAX_TOKENS = 16;   // tokens per verify block (rows per expert problem <= 16)
constexpr int MAX_K = 16;

// One CTA.  Table layout (int32): [0] = P (active experts); [1 .. E] active
// expert ids in increasing order; [1+E .. 1+2E) rows per problem;
// [1+2E ..) token of row m of problem pi at (pi * 16 + m); then E * 16 pair
// rows (t * k + j) in the same order.
__global__ void route_kernel(const float* logits, int T, int E, int k, int32_t* table,
                             float* weights, int32_t* topk) {
  extern __shared__ int sh[];
  int* cnt = sh;                 // [E]
  int* start = cnt + E;          // [E]
  int* ids = start + E;          // [T * k]
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  // top-k per token: one warp per token
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  for (int t = warp; t < T; t += nwarps) {
    const float* row = logits + (size_t)t * E;
    float kept[MAX_K];
    int kept_id[MAX_K];
    for (int j = 0; j < k; ++j) {
      // best not-yet-taken (value desc, id asc)
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        bool taken = false;
        for (int q = 0; q < j; ++q) taken |= (kept_id[q] == e);
        if (taken) continue;
        const float v = row[e];
        if (v > bv || (v == bv && e < bi)) { bv = v; bi = e; }
      }
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      kept[j] = bv;
      kept_id[j] = bi;
    }
    if (lane == 0) {
      float mx = kept[0];
      double den = 0.0;
      for (int j = 0; j < k; ++j) den += exp((double)kept[j] - mx);
      for (int j = 0; j < k; ++j) {
        weights[t * k + j] = float(exp((double)kept[j] - mx) / den);
        topk[t * k + j] = kept_id[j];
        ids[t * k + j] = kept_id[j];
        atomicAdd(&cnt[kept_id[j]], 1);
      }
    }
  }
  __syncthreads();
  // Active experts in increasing id order (serial over E in shared memory).
  if (tid == 0) {
    int P = 0;
    for (int e = 0; e < E; ++e) start[e] = cnt[e] > 0 ? P++ : -1;
    table[0] = P;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const int pi = start[e];
    if (pi >= 0) {
      table[1 + pi] = e;
      table[1 + E + pi] = cnt[e];
    }
  }
  // Rows of each problem in token order (t ascending, then slot): pair pr
  // is row m of its expert's problem, m = number of earlier pairs routed to
  // the same expert.  Computed per pair in parallel (deterministic).
  const int pairs = T * k;
  for (int pr = tid; pr < pairs; pr += blockDim.x) {
    const int e = ids[pr];
    int m = 0;
    for (int q = 0; q < pr; ++q) m += (ids[q] == e);
    const int pi = start[e];
    table[1 + 2 * E + pi * 16 + m] = pr / k;          // token row
    table[1 + 2 * E + 16 * E + pi * 16 + m] = pr;     // pair row
  }
}

__global__ void silu_mul_kernel(const uint16_t* gate, const uint16_t* up, uint16_t* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = silu_mul_bits<false>(gate[i], up[i]);
}

// Same on row-strided inputs: out[r, c] (contiguous) from gate/up rows of
// stride ld, e.g. the two halves of a fused gate|up projection output.
// Launched with programmatic stream serialization, like the qmm it sits
// between: it lets the next launch start its weight prefetch at once and
// waits for the previous launch's output before reading it.
__global__ void silu_mul_rows_kernel(const uint16_t* gate, const uint16_t* up, int ld, uint16_t* out,
                                     int rows, int cols) {
  griddep_launch_dependents();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int r = i / cols, c = i - r * cols;
  const size_t j = (size_t)r * ld + c;
  out[i] = silu_mul_bits<false>(gate[j], up[j]);
}

// y[t, c] = bf16( sum_j w[t, j] * pair_out[t * k + j, c]  (+ shared[t, c]) ), fp32 in slot order
__global__ void combine_kernel(const uint16_t* pair_out, const float* weights, const uint16_t* shared,
                               uint16_t* y, int T, int k, int H) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * H) return;
  const int t = i / H, c = i - t * H;
  float acc = 0.f;
  for (int j = 0; j < k; ++j) {
    const float v = __bfloat162float(__ushort_as_bfloat16(pair_out[((size_t)t * k + j) * H + c]));
    acc = __fadd_rn(acc, __fmul_rn(weights[t * k + j], v));
  }
  if (shared) acc = __fadd_rn(acc, __bfloat162float(__ushort_as_bfloat16(shared[i])));
  y[i] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
}

// Sorted route table of grouped plan phases (qmm_plan.cu) from the top-k
// expert ids, plus the x rows in sorted order.  Sorted rows are the (token,
// slot) pairs ordered by expert id, then pair index (= token order, then
// slot, as route_kernel numbers a problem's rows).  Every CTA ranks all
// pairs in shared memory (pairs <= 256); CTA 0 writes the table, and the
// CTAs share the row copies.
//   route[0] = P (active experts); route[1 + 2i] = first sorted row of
//   problem i (i <= P, route[1 + 2P] = pairs); route[2 + 2i] = its expert;
//   route[kRouteRowMap + r] = pair row of sorted row r.
// ex[] holds the pairs' expert ids (validated by the caller), first[] and
// pos[] are shared scratch of the same length.
// shared >= 0: one more problem after the routed ones, expert `shared`, whose
// rows are the T tokens themselves (sorted rows pairs .. pairs + T - 1, row
// map to pair rows pairs + t): a shared expert run as one more grouped problem.
__device__ void rank_and_gather(const int* ex, int* first, int* pos, int pairs, int top_k,
                                const uint16_t* x, int ldx, int H, int32_t* route,
                                uint16_t* x_sorted, uint16_t* x_copy, int T, int shared) {
  const int tid = threadIdx.x;
  for (int p = tid; p < pairs; p += blockDim.x) {
    int f = 1;
    for (int q = 0; q < p; ++q) f &= (ex[q] != ex[p]);
    first[p] = f;
  }
  __syncthreads();
  // rank of pair p: pairs with a smaller expert id, plus earlier pairs with
  // the same one; problem index of its expert: distinct smaller expert ids
  for (int p = tid; p < pairs; p += blockDim.x) {
    const int e = ex[p];
    int below = 0, same_before = 0, distinct_below = 0;
    for (int q = 0; q < pairs; ++q) {
      const int eq = ex[q];
      below += (eq < e);
      same_before += (eq == e && q < p);
      distinct_below += (eq < e) & first[q];
    }
    pos[p] = below + same_before;
    if (blockIdx.x == 0) {
      route[plan::kRouteRowMap + below + same_before] = p;
      if (first[p]) {
        route[1 + 2 * distinct_below] = below;
        route[2 + 2 * distinct_below] = e;
      }
    }
  }
  const int P = __syncthreads_count(tid < pairs && first[tid]);
  if (blockIdx.x == 0) {
    if (tid == 0) {
      route[1 + 2 * P] = pairs;
      if (shared >= 0) {
        route[0] = P + 1;
        route[2 + 2 * P] = shared;
        route[3 + 2 * P] = pairs + T;
      } else {
        route[0] = P;
      }
    }
    if (shared >= 0)
      for (int t = tid; t < T; t += blockDim.x) route[plan::kRouteRowMap + pairs + t] = pairs + t;
  }
  // rows: x_sorted[pos[p]] = x[p / top_k] (16-byte words), then the shared
  // expert's rows x_sorted[pairs + t] = x[t], then the caller's x copied
  // whole into x_copy, by the same CTAs
  const int words = H / 8;
  const int n_shared = shared >= 0 ? T : 0;
  const int jobs = pairs + n_shared + (x_copy ? T : 0);
  for (int j = blockIdx.x; j < jobs; j += gridDim.x) {
    const uint4* src;
    uint4* dst;
    if (j < pairs) {
      src = reinterpret_cast<const uint4*>(x + size_t(j / top_k) * ldx);
      dst = reinterpret_cast<uint4*>(x_sorted + size_t(pos[j]) * H);
    } else if (j < pairs + n_shared) {
      src = reinterpret_cast<const uint4*>(x + size_t(j - pairs) * ldx);
      dst = reinterpret_cast<uint4*>(x_sorted + size_t(j) * H);
    } else {
      src = reinterpret_cast<const uint4*>(x + size_t(j - pairs - n_shared) * ldx);
      dst = reinterpret_cast<uint4*>(x_copy + size_t(j - pairs - n_shared) * H);
    }
    for (int i = tid; i < words; i += blockDim.x) dst[i] = src[i];
  }
}

// An expert id outside [0, E) sets the device error word and the table gets
// P = 0 (grouped phases then do nothing).
__global__ void sort_pairs_kernel(const int32_t* topk_ids, int pairs, int top_k, int E,
                                  const uint16_t* x, int ldx, int H, int32_t* route,
                                  uint16_t* x_sorted, uint16_t* x_copy, int T) {
  __shared__ int ex[plan::kRouteMaxRows];
  __shared__ int first[plan::kRouteMaxRows];   // pair p is its expert's first pair
  __shared__ int pos[plan::kRouteMaxRows];
  __shared__ int bad;
  const int tid = threadIdx.x;
  if (tid == 0) bad = 0;
  __syncthreads();
  for (int p = tid; p < pairs; p += blockDim.x) {
    const int e = topk_ids[p];
    ex[p] = e;
    if (e < 0 || e >= E) bad = 1;
  }
  __syncthreads();
  if (bad) {
    if (blockIdx.x == 0 && tid == 0) {
      atomicExch(&g_device_error, kDevBadInput);
      route[0] = 0;
      route[1] = 0;
    }
    return;
  }
  rank_and_gather(ex, first, pos, pairs, top_k, x, ldx, H, route, x_sorted, x_copy, T, -1);
}

constexpr int kRouteSortMaxExperts = 4096;

// (value desc, id asc): the order in which experts are picked
__device__ __forceinline__ bool beats(float v, int e, float w, int f) {
  return v > w || (v == w && e < f);
}

// Routing and sorting in one launch (MoEPlanLayer): warp t takes token t's
// top-k by router logit (largest first, ties to the lower id: each lane
// keeps a best-first list of its own experts e = lane + 32 i in registers,
// then k rounds of a warp argmax over the lanes' heads pick the experts in
// route_kernel's order) and its softmax over the kept logits in double
// precision (the same operations as route_kernel, so the same weights bit
// for bit); CTA 0 stores weights and ids; then every CTA ranks the pairs and
// copies its share of the rows (rank_and_gather).  A top-k with no winner
// (NaN logits) sets the device error word and the table gets P = 0.
__global__ void route_sort_kernel(const float* logits, int T, int E, int k, int shared,
                                  const uint16_t* x, int ldx, int H, int32_t* route, float* weights,
                                  int32_t* topk, uint16_t* x_sorted, uint16_t* x_copy) {
  __shared__ int ex[plan::kRouteMaxRows];
  __shared__ int first[plan::kRouteMaxRows];
  __shared__ int pos[plan::kRouteMaxRows];
  __shared__ int bad;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) bad = 0;
  __syncthreads();
  if (warp < T) {
    const int t = warp;
    const float* row = logits + (size_t)t * E;
    float lv[MAX_K];
    int li[MAX_K];
#pragma unroll
    for (int i = 0; i < MAX_K; ++i) {
      lv[i] = -INFINITY;
      li[i] = 0x7fffffff;
    }
    // this lane's logits, 8 loads in flight at a time
    for (int e0 = lane; e0 < E; e0 += 32 * 8) {
      float vb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) vb[u] = (e0 + 32 * u < E) ? row[e0 + 32 * u] : -INFINITY;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + 32 * u;
        const float v = vb[u];
        if (e >= E || !beats(v, e, lv[MAX_K - 1], li[MAX_K - 1])) continue;
        // insertion from the tail: entries (v, e) beats move down one place
#pragma unroll
        for (int i = MAX_K - 1; i >= 1; --i) {
          if (beats(v, e, lv[i], li[i])) {
            const bool above = beats(v, e, lv[i - 1], li[i - 1]);
            lv[i] = above ? lv[i - 1] : v;
            li[i] = above ? li[i - 1] : e;
          }
        }
        if (beats(v, e, lv[0], li[0])) {
          lv[0] = v;
          li[0] = e;
        }
      }
    }
    float myv = 0.f;
    int myid = 0;
    for (int j = 0; j < k; ++j) {
      float bv = lv[0];
      int bi = li[0];
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (beats(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (lane == j) {
        myv = bv;
        myid = bi;
      }
      if (bi < 0 || bi >= E) {
        if (lane == 0) bad = 1;
        break;
      }
      if (li[0] == bi) {
        // this lane's head was picked: pop it
#pragma unroll
        for (int i = 0; i < MAX_K - 1; ++i) {
          lv[i] = lv[i + 1];
          li[i] = li[i + 1];
        }
        lv[MAX_K - 1] = -INFINITY;
        li[MAX_K - 1] = 0x7fffffff;
      }
    }
    const float mx = __shfl_sync(0xffffffffu, myv, 0);
    const double v = (lane < k) ? exp((double)myv - mx) : 0.0;
    double den = 0.0;
    for (int j = 0; j < k; ++j) den += __shfl_sync(0xffffffffu, v, j);
    if (lane < k) {
      ex[t * k + lane] = myid;
      if (blockIdx.x == 0) {
        weights[t * k + lane] = float(v / den);
        topk[t * k + lane] = myid;
      }
    }
  }
  __syncthreads();
  if (bad) {
    if (blockIdx.x == 0 && tid == 0) {
      atomicExch(&g_device_error, kDevBadInput);
      route[0] = 0;
      route[1] = 0;
    }
    return;
  }
  rank_and_gather(ex, first, pos, T * k, k, x, ldx, H, route, x_sorted, x_copy, T, shared);
}

}  // namespace moe
}  // namespace dfl

extern "C" int dfl_moe_route(const float* logits, int T, int E, int top_k, int32_t* route_table,
                             float* weights, int32_t* topk_ids, void* stream) {
  using namespace dfl;
  if (T < 1 || T > moe::MAX_TOKENS || E < 1 || E > 4096 || top_k < 1 || top_k > moe::MAX_K ||
      top_k > E)
    return DFL_ERR_BAD_SHAPE;
  if (!logits || !route_table || !weights || !topk_ids) return DFL_ERR_NULL_POINTER;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  const size_t smem = (2 * size_t(E) + size_t(T) * top_k) * sizeof(int);
  moe::route_kernel<<<1, 512, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, T, E, top_k, route_table, weights, topk_ids);
  return host::launch_status();
}

extern "C" size_t dfl_moe_route_table_ints(int E) { return 1 + 2 * size_t(E) + 32 * size_t(E); }

extern "C" int dfl_silu_mul_bf16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int n,
                                 void* stream) {
  using namespace dfl;
  if (n < 0) return DFL_ERR_BAD_SHAPE;
  if (n == 0) return DFL_OK;
  if (!gate || !up || !out) return DFL_ERR_NULL_POINTER;
  moe::silu_mul_kernel<<<(n + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      gate, up, out, n);
  return host::launch_status();
}

extern "C" int dfl_silu_mul_rows_bf16(const uint16_t* gate, const uint16_t* up, int ld,
                                      uint16_t* out, int rows, int cols, void* stream) {
  using namespace dfl;
  if (rows < 0 || cols < 0 || ld < cols) return DFL_ERR_BAD_SHAPE;
  if ((long long)rows * cols > 0x7fffffffLL) return DFL_ERR_BAD_SHAPE;
  if (rows == 0 || cols == 0) return DFL_OK;
  if (!gate || !up || !out) return DFL_ERR_NULL_POINTER;
  const int n = rows * cols;
  return host::launch_pdl(moe::silu_mul_rows_kernel, (n + 255) / 256, 256, 0,
                          reinterpret_cast<cudaStream_t>(stream), gate, up, ld, out, rows, cols);
}

extern "C" int dfl_moe_combine(const uint16_t* pair_out, const float* weights,
                               const uint16_t* shared, uint16_t* y, int T, int top_k, int H,
                               void* stream) {
  using namespace dfl;
  if (T < 0 || top_k < 1 || H < 1) return DFL_ERR_BAD_SHAPE;
  if (T == 0) return DFL_OK;
  if (!pair_out || !weights || !y) return DFL_ERR_NULL_POINTER;
  const int n = T * H;
  moe::combine_kernel<<<(n + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      pair_out, weights, shared, y, T, top_k, H);
  return host::launch_status();
}

extern "C" size_t dfl_moe_sorted_route_ints(void) { return size_t(dfl::plan::kRouteInts); }

extern "C" int dfl_moe_sort_pairs(const int32_t* topk_ids, int T, int top_k, int E,
                                  const uint16_t* x, int ldx, int H, int32_t* route,
                                  uint16_t* x_sorted, uint16_t* x_copy, void* stream) {
  using namespace dfl;
  if (T < 1 || top_k < 1 || (long long)T * top_k > plan::kRouteMaxRows || E < 1 || E > (1 << 20) ||
      H < 8 || H % 8 != 0 || ldx < H || ldx % 8 != 0)
    return DFL_ERR_BAD_SHAPE;
  if (!topk_ids || !x || !route || !x_sorted) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(topk_ids, 4) || !host::aligned(route, 4) || !host::aligned(x, 16) ||
      !host::aligned(x_sorted, 16) || (x_copy && !host::aligned(x_copy, 16)))
    return DFL_ERR_MISALIGNED;
  const int pairs = T * top_k;
  const int blocks = pairs + (x_copy ? T : 0) < 64 ? pairs + (x_copy ? T : 0) : 64;
  moe::sort_pairs_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      topk_ids, pairs, top_k, E, x, ldx, H, route, x_sorted, x_copy, T);
  return host::launch_status();
}

extern "C" int dfl_moe_route_sorted(const float* logits, int T, int E, int top_k, int shared_expert,
                                    const uint16_t* x, int ldx, int H, int32_t* route, float* weights,
                                    int32_t* topk_ids, uint16_t* x_sorted, uint16_t* x_copy,
                                    void* stream) {
  using namespace dfl;
  if (T < 1 || T > moe::MAX_TOKENS || E < 1 || E > moe::kRouteSortMaxExperts || top_k < 1 ||
      top_k > moe::MAX_K || top_k > E || T * top_k + (shared_expert ? T : 0) > plan::kRouteMaxRows ||
      H < 8 || H % 8 != 0 || ldx < H || ldx % 8 != 0 || (shared_expert != 0 && shared_expert != 1))
    return DFL_ERR_BAD_SHAPE;
  if (!logits || !x || !route || !weights || !topk_ids || !x_sorted) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(logits, 4) || !host::aligned(route, 4) || !host::aligned(weights, 4) ||
      !host::aligned(topk_ids, 4) || !host::aligned(x, 16) || !host::aligned(x_sorted, 16) ||
      (x_copy && !host::aligned(x_copy, 16)))
    return DFL_ERR_MISALIGNED;
  const int jobs = T * top_k + (shared_expert ? T : 0) + (x_copy ? T : 0);
  const int blocks = jobs < 148 ? jobs : 148;
  moe::route_sort_kernel<<<blocks, 512, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, T, E, top_k, shared_expert ? E : -1, x, ldx, H, route, weights, topk_ids, x_sorted,
      x_copy);
  return host::launch_status();
}
