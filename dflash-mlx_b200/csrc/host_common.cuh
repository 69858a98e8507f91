// Host-side helpers shared by the C-ABI entry points: status codes, device
// property caches, tensor-map encoding through the driver entry point
// (so the library does not link libcuda and loads on machines without a
// GPU), and per-kernel shared-memory opt-in.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "../../include/dflash_b200.h"

namespace dfl {
namespace host {

constexpr int kMaxDevices = 64;

// Every workspace starts with this many bytes of counters that are zero
// between calls (each kernel resets what it uses); kernels put their other
// scratch data after it, so one buffer can serve any sequence of calls.
constexpr size_t kWorkspaceCounterBytes = 64 * 1024;

struct DeviceInfo {
  std::atomic<int> num_sms{0};
  std::atomic<int> cc_major{0};
};

inline DeviceInfo& device_info(int dev) {
  static DeviceInfo infos[kMaxDevices];
  return infos[dev];
}

// Current device, its SM count and a check that it is an sm_100 part.
inline int current_device(int* dev_out, int* num_sms_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DFL_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return DFL_ERR_UNSUPPORTED;
  DeviceInfo& info = device_info(dev);
  int sms = info.num_sms.load(std::memory_order_acquire);
  int major = info.cc_major.load(std::memory_order_acquire);
  if (sms == 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return DFL_ERR_CUDA;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return DFL_ERR_CUDA;
    info.cc_major.store(major, std::memory_order_release);
    info.num_sms.store(sms, std::memory_order_release);
  }
  if (major != 10) return DFL_ERR_UNSUPPORTED;
  *dev_out = dev;
  *num_sms_out = sms;
  return DFL_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major tensor map: dims {inner, outer}, row stride in bytes,
// box {box_inner, box_outer}.  Out-of-range elements read as zero.
inline int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                        uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                        uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return DFL_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return DFL_ERR_MISALIGNED;
  if (row_stride_bytes % 16 != 0) return DFL_ERR_MISALIGNED;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DFL_OK : DFL_ERR_CUDA;
}

// 3-D tensor map: dims {inner, outer, depth}, strides in bytes for the two
// outer dims, box {box_inner, box_outer, 1}.  Out-of-range elements read as 0.
inline int make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                        uint64_t inner, uint64_t outer, uint64_t depth, uint64_t outer_stride_bytes,
                        uint64_t depth_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return DFL_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return DFL_ERR_MISALIGNED;
  if (outer_stride_bytes % 16 != 0 || depth_stride_bytes % 16 != 0) return DFL_ERR_MISALIGNED;
  cuuint64_t dims[3] = {inner, outer, depth};
  cuuint64_t strides[2] = {outer_stride_bytes, depth_stride_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DFL_OK : DFL_ERR_CUDA;
}

// Opt a kernel into `bytes` of dynamic shared memory once per device.
template <typename Kernel>
inline int ensure_smem(Kernel kernel, int bytes, int dev, std::atomic<uint64_t>& done_mask) {
  const uint64_t bit = uint64_t(1) << dev;
  if (done_mask.load(std::memory_order_acquire) & bit) return DFL_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return DFL_ERR_CUDA;
  done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return DFL_OK;
}

// Launch with programmatic stream serialization: the kernel may begin (its
// prologue and its weight loads) while the previous kernel in the stream is
// still running; it calls griddep_wait() before touching that kernel's outputs.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), int grid, int block, size_t smem,
                      cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) != cudaSuccess) {
    cudaGetLastError();
    return DFL_ERR_CUDA;
  }
  return DFL_OK;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DFL_OK : DFL_ERR_CUDA;
}

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

}  // namespace host
}  // namespace dfl
