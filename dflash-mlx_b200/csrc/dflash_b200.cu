// Single translation unit of libdflash_b200.so: the device error word, the
// generic C-ABI helpers and every kernel family (one TU keeps device
// symbols private without relocatable device code).
#include "common.cuh"
#include "host_common.cuh"

#include "qmm_w4.cu"
#include "qmm_noalloc.cu"
#include "qmm_plan.cu"
#include "gdn_replay.cu"
#include "gdn_forward.cu"
#include "gdn_tree.cu"
#include "lmhead.cu"
#include "moe.cu"

extern "C" const char* dfl_status_string(int status) {
  switch (status) {
    case DFL_OK: return "ok";
    case DFL_ERR_NULL_POINTER: return "null pointer";
    case DFL_ERR_BAD_SHAPE: return "unsupported shape";
    case DFL_ERR_MISALIGNED: return "misaligned pointer or stride";
    case DFL_ERR_WORKSPACE: return "workspace missing or too small";
    case DFL_ERR_CUDA: return "CUDA error";
    case DFL_ERR_UNSUPPORTED: return "unsupported device or option";
    case DFL_ERR_SCRATCH_LIMIT: return "shape needs more scratch than the fixed no-allocation array";
    default: return "unknown status";
  }
}

extern "C" const char* dfl_version(void) { return "dflash-b200 0.1.0 (sm_100a)"; }

extern "C" int dfl_get_device_error(int* device_error) {
  if (!device_error) return DFL_ERR_NULL_POINTER;
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return DFL_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&v, dfl::g_device_error, sizeof(int)) != cudaSuccess) return DFL_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(dfl::g_device_error, &zero, sizeof(int)) != cudaSuccess) return DFL_ERR_CUDA;
  if (v != 0) {
    // a timed-out qmm may have left partial sums in the no-allocation scratch
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DFL_ERR_CUDA;
    const int st = dfl::qmm_noalloc::reset_after_device_error(dev);
    if (st != DFL_OK) return st;
  }
  *device_error = v;
  return DFL_OK;
}
