// lm_head verify epilogue: argmax of h @ W^T over the vocabulary without
// writing logits, then greedy acceptance.
//
// Replaces, for the verify block, logits_from_hidden
// (dflash_mlx/engine/target_qwen_gdn.py:774-778: embed_tokens.as_linear or
// lm_head, bf16 logits), greedy_tokens_with_mask
// (dflash_mlx/engine/sampling.py:47-55: suppressed ids get the bf16 floor
// -1e9, then the first index of the maximum) and match_acceptance_length
// (dflash_mlx/engine/acceptance.py:9-16) as composed at
// dflash_mlx/engine/spec_epoch.py:2067-2072,2129.
//
// Kernel 1 (persistent, swap-AB tcgen05 GEMM): a work unit is one 128-row
// vocabulary tile (the UMMA M dimension, rows = TMEM lanes) against up to
// RT = 16..256 hidden rows (the UMMA N dimension).  TMA streams the bf16
// weight tile and the hidden rows per 64-wide K block (128-byte swizzle)
// through a shared-memory ring; one thread issues the MMAs into a
// double-buffered fp32 TMEM accumulator; four epilogue warps read it back
// (tcgen05.ld), round each logit to bf16 (the reference's logits dtype),
// apply the suppress mask and fold (value, vocabulary id) into one 64-bit
// key per hidden row: high word an order-preserving image of the value, low
// word ~id, so the maximum key is the maximum logit with ties going to the
// lowest id -- exactly argmax's "first index" rule.  Keys are reduced with a
// warp shuffle max and a shared-memory atomicMax per row; each CTA writes its
// per-row keys, and the last CTA to finish (atomic counter) reduces them.
// Logits never leave the chip.
//
// Kernel 2 (accept): reduces the keys of G vocabulary shards (G > 1 after an
// all-gather), decodes posterior tokens and runs the acceptance scan on
// device, so the host reads back only ids and lengths.
#include "common.cuh"
#include "host_common.cuh"

namespace dfl {
namespace lmh {

constexpr int BV = 128;        // vocabulary rows per tile (UMMA M)
constexpr int BK = 64;         // K per stage (one 128-byte swizzle atom)
constexpr int NUM_THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr int WARP_EPI0 = 2;
constexpr int MAX_ROWS = 4096;    // hidden rows per call (running keys in shared memory)
constexpr size_t kCounterBytes = host::kWorkspaceCounterBytes;

template <int RT>
struct Cfg {
  static constexpr int A_BYTES = BV * BK * 2;      // 16 KB
  static constexpr int B_BYTES = RT * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NSTAGE = (RT <= 64) ? 8 : (RT <= 128 ? 6 : 4);
  static constexpr int TMEM_COLS = (2 * RT < 32) ? 32 : 2 * RT;
  static constexpr int OFF_KEYS = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_BARS = OFF_KEYS + MAX_ROWS * 8;
  static constexpr int SMEM_BYTES = OFF_BARS + 256 + 1024;
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

struct Params {
  const uint8_t* suppress;   // [V_total] or null, indexed by global id
  unsigned long long* out_keys;  // [R]
  unsigned long long* row_max;   // workspace [R]: running key maximum per row, zero between calls
  int* counter;
  int R, D, V, v_begin;
  int n_vtiles, n_rg, units, grid;
};

// Order-preserving image of a float in 32 bits (larger float -> larger word).
// -0 is folded into +0 first (x + 0 is +0 for both zeros under round-to-
// nearest), so equal logits always tie and the lower id wins, as in argmax.
__host__ __device__ __forceinline__ uint32_t ordered_bits(float v) {
  v = v + 0.0f;
#ifdef __CUDA_ARCH__
  const uint32_t u = __float_as_uint(v);
#else
  uint32_t u;
  std::memcpy(&u, &v, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ unsigned long long make_key(float v, uint32_t id) {
  return (static_cast<unsigned long long>(ordered_bits(v)) << 32) | (0xFFFFFFFFu - id);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
    k = o > k ? o : k;
  }
  return k;
}

template <int RT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    lmhead_argmax_kernel(const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_h, const Params p) {
  using C = Cfg<RT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem + C::OFF_KEYS);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BARS);
  uint64_t* empty = full + C::NSTAGE;
  uint64_t* accfull = empty + C::NSTAGE;   // [2]
  uint64_t* accempty = accfull + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(flag + 1);
  auto wait = [abort_word](uint64_t* bar, uint32_t parity) {
    return mbar_wait_abortable(bar, parity, abort_word);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblocks = (p.D + BK - 1) / BK;

  for (int i = threadIdx.x; i < p.R; i += NUM_THREADS) keys[i] = 0ull;
  if (threadIdx.x == 0) {
    *abort_word = 0;
    for (int i = 0; i < C::NSTAGE; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_h);
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += p.grid) {
        const int vt = u / p.n_rg, rg = u - vt * p.n_rg;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % C::NSTAGE;
          if (!wait(&empty[s], ((it / C::NSTAGE) & 1) ^ 1)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(st, &tm_w, &full[s], kb * BK, vt * BV);
          tma_load_2d(st + C::A_BYTES, &tm_h, &full[s], kb * BK, rg * RT);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BV, RT);
      int it = 0, ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += p.grid, ++ui) {
        const uint32_t buf = ui & 1;
        if (!wait(&accempty[buf], ((ui >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * RT;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % C::NSTAGE;
          if (!wait(&full[s], (it / C::NSTAGE) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t adesc = make_sw128_desc(a);
          const uint64_t bdesc = make_sw128_desc(a + C::A_BYTES);
          mma_bf16_ss(d_tmem, adesc, bdesc, idesc, kb > 0 ? 1u : 0u);
          mma_bf16_ss(d_tmem, adesc + 2, bdesc + 2, idesc, 1u);
          mma_bf16_ss(d_tmem, adesc + 4, bdesc + 4, idesc, 1u);
          mma_bf16_ss(d_tmem, adesc + 6, bdesc + 6, idesc, 1u);
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&accfull[buf]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;      // vocabulary row within the tile
    const uint32_t lane_base = tmem_base + (uint32_t(quad * 32) << 16);
    const float floor_v = __bfloat162float(__float2bfloat16_rn(-1e9f));
    int ui = 0;
    for (int u = blockIdx.x; u < p.units; u += p.grid, ++ui) {
      const int vt = u / p.n_rg, rg = u - vt * p.n_rg;
      const uint32_t buf = ui & 1;
      if (!wait(&accfull[buf], (ui >> 1) & 1)) break;
      tc_fence_after();
      const int vloc = vt * BV + row;
      const bool valid = vloc < p.V;
      const uint32_t gid = uint32_t(p.v_begin + vloc);
      const bool suppressed = valid && p.suppress && p.suppress[gid];
#pragma unroll 1
      for (int c0 = 0; c0 < RT; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(lane_base + buf * RT + c0, r);
        tmem_ld_wait();
        if (c0 + 16 >= RT) {
          // accumulator fully read: hand it back to the MMA issuer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[buf]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float v = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[i])));
          if (suppressed) v = floor_v;
          unsigned long long key = valid ? make_key(v, gid) : 0ull;
          key = warp_max_u64(key);
          const int hr = rg * RT + c0 + i;
          if (lane == 0 && hr < p.R) atomicMax(&keys[hr], key);
        }
      }
    }
  }

  // fold this CTA's row keys into the workspace's running maxima; the last
  // CTA copies them out and zeroes them again, so the workspace is all zero
  // when the kernel ends (the convention every workspace user relies on:
  // one buffer serves any sequence of calls on a stream)
  tc_fence_before();
  __syncthreads();
  for (int i = threadIdx.x; i < p.R; i += NUM_THREADS) {
    const unsigned long long k = keys[i];
    if (k != 0ull) atomicMax(&p.row_max[i], k);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *flag = (atomicAdd(p.counter, 1) == p.grid - 1) ? 1 : 0;
  __syncthreads();
  if (*flag) {
    __threadfence();
    for (int i = threadIdx.x; i < p.R; i += NUM_THREADS) {
      p.out_keys[i] = __ldcg(&p.row_max[i]);
      __stcg(&p.row_max[i], 0ull);
    }
    if (threadIdx.x == 0) *p.counter = 0;
  }
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// Accept: keys [G][B*T] -> posterior [B][T], acceptance [B], next token [B].
// acceptance = sum_i prod_{j<=i} [verify_ids[b, j+1] == posterior[b, j]]
// (engine/acceptance.py:9-16 applied to verify_ids[1:] vs posterior[:-1]);
// next token = posterior[b, acceptance] (engine/spec_epoch.py:2129).
__global__ void accept_kernel(const unsigned long long* keys, int G, const int32_t* verify_ids,
                              int B, int T, int32_t* posterior, int32_t* acceptance,
                              int32_t* next_token, float* max_logit) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int R = B * T;
  int acc = 0;
  bool run = true;
  for (int t = 0; t < T; ++t) {
    unsigned long long best = 0ull;
    for (int g = 0; g < G; ++g) {
      const unsigned long long k = keys[(size_t)g * R + (size_t)b * T + t];
      best = k > best ? k : best;
    }
    const int32_t id = int32_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFull));
    posterior[(size_t)b * T + t] = id;
    if (max_logit) {
      uint32_t hi = uint32_t(best >> 32);
      const uint32_t u = (hi & 0x80000000u) ? (hi & 0x7FFFFFFFu) : ~hi;
      max_logit[(size_t)b * T + t] = __uint_as_float(u);
    }
    if (verify_ids && run && t + 1 < T) {
      if (verify_ids[(size_t)b * T + t + 1] == id) ++acc;
      else run = false;
    }
  }
  if (acceptance) acceptance[b] = acc;
  if (next_token) {
    // posterior[acc] (acc <= T - 1)
    next_token[b] = posterior[(size_t)b * T + acc];
  }
}

// acceptance[b] = sum_i prod_{j<=i} [drafted[b, j] == posterior[b, j]]
// (engine/acceptance.py:9-16), for B rows of length L.
__global__ void match_acceptance_kernel(const int32_t* drafted, const int32_t* posterior, int B,
                                        int L, int32_t* out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int acc = 0;
  while (acc < L && drafted[(size_t)b * L + acc] == posterior[(size_t)b * L + acc]) ++acc;
  out[b] = acc;
}

inline int choose_rt(int R) {
  if (R <= 16) return 16;
  if (R <= 32) return 32;
  if (R <= 64) return 64;
  if (R <= 128) return 128;
  return 256;
}

inline void geometry(int R, int V, int num_sms, int* n_vtiles, int* n_rg, int* units, int* grid) {
  const int rt = choose_rt(R);
  *n_vtiles = (V + BV - 1) / BV;
  *n_rg = (R + rt - 1) / rt;
  *units = *n_vtiles * *n_rg;
  *grid = *units < num_sms ? *units : num_sms;
}

inline size_t workspace_bytes_for(int R, int V, int num_sms) {
  int nv, nrg, units, grid;
  geometry(R, V, num_sms, &nv, &nrg, &units, &grid);
  (void)nv; (void)nrg; (void)units; (void)grid;
  return kCounterBytes + size_t(R) * sizeof(unsigned long long);
}

template <int RT>
int launch(const uint16_t* h, const uint16_t* w, int R, int D, int V, int v_begin,
           const uint8_t* suppress, unsigned long long* out_keys, void* ws, int num_sms, int dev,
           cudaStream_t stream) {
  using C = Cfg<RT>;
  static std::atomic<uint64_t> done{0};
  int st = host::ensure_smem(lmhead_argmax_kernel<RT>, C::SMEM_BYTES, dev, done);
  if (st != DFL_OK) return st;
  Params p;
  p.suppress = suppress;
  p.out_keys = out_keys;
  p.counter = reinterpret_cast<int*>(ws);
  p.row_max = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(ws) + kCounterBytes);
  p.R = R;
  p.D = D;
  p.V = V;
  p.v_begin = v_begin;
  geometry(R, V, num_sms, &p.n_vtiles, &p.n_rg, &p.units, &p.grid);
  CUtensorMap tm_w, tm_h;
  st = host::make_tmap_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, uint64_t(D), uint64_t(V),
                          uint64_t(D) * 2, BK, BV, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != DFL_OK) return st;
  st = host::make_tmap_2d(&tm_h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, h, uint64_t(D), uint64_t(R),
                          uint64_t(D) * 2, BK, RT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != DFL_OK) return st;
  lmhead_argmax_kernel<RT><<<p.grid, NUM_THREADS, C::SMEM_BYTES, stream>>>(tm_w, tm_h, p);
  return host::launch_status();
}

}  // namespace lmh
}  // namespace dfl

extern "C" size_t dfl_lmhead_workspace_bytes(int R, int D, int V, int* status) {
  int dummy;
  int* st = status ? status : &dummy;
  if (R < 1 || R > dfl::lmh::MAX_ROWS || D < 8 || D % 8 != 0 || V < 1) {
    *st = DFL_ERR_BAD_SHAPE;
    return 0;
  }
  int dev, sms;
  *st = dfl::host::current_device(&dev, &sms);
  if (*st != DFL_OK) return 0;
  return dfl::lmh::workspace_bytes_for(R, V, sms);
}

extern "C" int dfl_lmhead_argmax(const uint16_t* h, const uint16_t* w, int R, int D, int V,
                                 int v_begin, const uint8_t* suppress, uint64_t* keys,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  using namespace dfl;
  if (R < 1 || R > lmh::MAX_ROWS || D < 8 || D % 8 != 0 || V < 1 || v_begin < 0)
    return DFL_ERR_BAD_SHAPE;
  if (!h || !w || !keys) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(h, 16) || !host::aligned(w, 16) || !host::aligned(keys, 8))
    return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  if (!workspace || workspace_bytes < lmh::workspace_bytes_for(R, V, sms)) return DFL_ERR_WORKSPACE;
  if (!host::aligned(workspace, 16)) return DFL_ERR_MISALIGNED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned long long* k = reinterpret_cast<unsigned long long*>(keys);
  switch (lmh::choose_rt(R)) {
    case 16: return lmh::launch<16>(h, w, R, D, V, v_begin, suppress, k, workspace, sms, dev, s);
    case 32: return lmh::launch<32>(h, w, R, D, V, v_begin, suppress, k, workspace, sms, dev, s);
    case 64: return lmh::launch<64>(h, w, R, D, V, v_begin, suppress, k, workspace, sms, dev, s);
    case 128: return lmh::launch<128>(h, w, R, D, V, v_begin, suppress, k, workspace, sms, dev, s);
    default: return lmh::launch<256>(h, w, R, D, V, v_begin, suppress, k, workspace, sms, dev, s);
  }
}

extern "C" int dfl_lmhead_accept(const uint64_t* keys, int G, const int32_t* verify_ids, int B,
                                 int T, int32_t* posterior, int32_t* acceptance,
                                 int32_t* next_token, float* max_logit, void* stream) {
  using namespace dfl;
  if (G < 1 || B < 0 || T < 1) return DFL_ERR_BAD_SHAPE;
  if (B == 0) return DFL_OK;
  if (!keys || !posterior) return DFL_ERR_NULL_POINTER;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  lmh::accept_kernel<<<(B + 127) / 128, 128, 0, s>>>(
      reinterpret_cast<const unsigned long long*>(keys), G, verify_ids, B, T, posterior,
      acceptance, next_token, max_logit);
  return host::launch_status();
}

extern "C" int dfl_match_acceptance(const int32_t* drafted, const int32_t* posterior, int B, int L,
                                    int32_t* acceptance, void* stream) {
  using namespace dfl;
  if (B < 0 || L < 0) return DFL_ERR_BAD_SHAPE;
  if (B == 0) return DFL_OK;
  if (!acceptance || (L > 0 && (!drafted || !posterior))) return DFL_ERR_NULL_POINTER;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  lmh::match_acceptance_kernel<<<(B + 127) / 128, 128, 0, s>>>(drafted, posterior, B, L, acceptance);
  return host::launch_status();
}
