// Dense int4 g64 verify qmm for callers that cannot allocate device memory.
//
// Same kernel and arguments as dfl_verify_qmm_w4g64, but the split-K scratch
// (fp32 partial sums) lives in one fixed file-scope device
// array instead of a caller workspace:
//   * kScratchBytes (8 MiB) is the limit; a call whose scratch need
//     (dfl_verify_qmm_workspace_bytes for its shape) is larger returns
//     DFL_ERR_SCRATCH_LIMIT.  For M <= 32 the need is 64 KB + 16 KB per CTA
//     (at most 160 CTAs), at most 2.6 MB (B200: 148 CTAs -> 2.4 MB).
//   * The first call on a device resolves the array's address on that
//     device (cudaGetSymbolAddress, with that device current); make it
//     before any stream capture on that device.
//   * Every call on a device shares the one array.  The first call on a
//     device zero-fills it on its stream; each kernel clears the partial
//     slots it consumes, so the array is zero again for the next call and
//     calls in stream order are safe; calls that may overlap in time
//     (different streams or host threads) race on the array.
//   * A call that timed out (device error word set) can leave partial sums
//     behind.  dfl_get_device_error, which synchronises the device, zero-fills
//     the array again on that device whenever it finds the word set, so
//     calls after that check are correct again.
// Nothing here calls cudaMalloc / cudaFree or any allocating routine.

namespace dfl {
namespace qmm_noalloc {

constexpr size_t kScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// The largest need of any accepted shape (M <= 32: tiles of 32 rows, at most
// kMaxGrid CTAs) fits, so DFL_ERR_SCRATCH_LIMIT is only a guard against a
// future change of the tile or grid constants.
static_assert(qmm::kCounterBytes + size_t(qmm::kMaxGrid) * 32 * qmm::BN * sizeof(float) <=
                  kScratchBytes,
              "the fixed scratch array must hold the split-K slots of every accepted shape");

struct DeviceScratch {
  std::atomic<void*> ptr{nullptr};
};

inline DeviceScratch& scratch_slot(int dev) {
  static DeviceScratch slots[host::kMaxDevices];
  return slots[dev];
}

// Device address of g_scratch on `dev` (the current device); resolved once,
// and zero-filled on `stream` by the first call.
inline int scratch_for_device(int dev, cudaStream_t stream, void** out) {
  DeviceScratch& slot = scratch_slot(dev);
  void* p = slot.ptr.load(std::memory_order_acquire);
  if (!p) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    p = slot.ptr.load(std::memory_order_acquire);
    if (!p) {
      if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return DFL_ERR_CUDA;
      }
      if (cudaMemsetAsync(p, 0, kScratchBytes, stream) != cudaSuccess) {
        cudaGetLastError();
        return DFL_ERR_CUDA;
      }
      slot.ptr.store(p, std::memory_order_release);
    }
  }
  *out = p;
  return DFL_OK;
}

// After a device error on `dev` (the current device, already synchronised):
// zero the array again if this device has resolved it, since a timed-out
// kernel may have left tagged partial sums in it.  Allocates nothing.
inline int reset_after_device_error(int dev) {
  if (dev < 0 || dev >= host::kMaxDevices) return DFL_OK;
  void* p = scratch_slot(dev).ptr.load(std::memory_order_acquire);
  if (!p) return DFL_OK;
  if (cudaMemset(p, 0, kScratchBytes) != cudaSuccess) {
    cudaGetLastError();
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

}  // namespace qmm_noalloc
}  // namespace dfl

extern "C" int dfl_verify_qmm_w4g64_noalloc(const uint16_t* x, const uint32_t* w_q,
                                            const uint16_t* scales, const uint16_t* biases,
                                            uint16_t* y, int M, int K, int N, void* stream) {
  using namespace dfl;
  if (M < 1 || M > 32 || K < 64 || K % 64 != 0 || N < 1 || N > qmm::kMaxTiles * qmm::BN)
    return DFL_ERR_BAD_SHAPE;
  if (!x || !w_q || !scales || !biases || !y) return DFL_ERR_NULL_POINTER;
  if (!host::aligned(x, 16) || !host::aligned(w_q, 16) || !host::aligned(scales, 2) ||
      !host::aligned(biases, 2) || !host::aligned(y, 2))
    return DFL_ERR_MISALIGNED;
  int dev, sms;
  int st = host::current_device(&dev, &sms);
  if (st != DFL_OK) return st;
  if (qmm::workspace_bytes_for(M, K, N, sms) > qmm_noalloc::kScratchBytes)
    return DFL_ERR_SCRATCH_LIMIT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  st = qmm_noalloc::scratch_for_device(dev, s, &scratch);
  if (st != DFL_OK) return st;
  if (qmm::choose_mt(M) == 16)
    return qmm::launch<16>(x, w_q, scales, biases, y, scratch, M, K, N, sms, dev, s);
  return qmm::launch<32>(x, w_q, scales, biases, y, scratch, M, K, N, sms, dev, s);
}
