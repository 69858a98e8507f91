/*
 * dflash-b200: C ABI of the B200-native target-verify hot path.
 *
 * Every entry point takes device pointers, plain sizes and a CUDA stream
 * (passed as void*; NULL means the legacy default stream), launches
 * asynchronously on that stream and returns a status code (DFL_OK == 0).
 * bf16 tensors are passed as uint16_t bit patterns.  Nothing here allocates
 * device memory; scratch memory is passed in by the caller.
 *
 * Reference interfaces replaced (paths inside the dflash-mlx project):
 *   dfl_verify_qmm_w4g64   <- verify_matmul            dflash_mlx/verify_qmm.py:905-1022
 *                             VerifyQuantizedLinear.__call__ dflash_mlx/verify_linear.py:115-116,266-286
 *                             (stock mx.quantized_matmul(transpose=True) for other M)
 *   dfl_gdn_tape_replay    <- tape_replay_kernel       dflash_mlx/kernels.py:822-868
 *   dfl_lmhead_argmax_partial + dfl_lmhead_accept
 *                          <- logits_from_hidden       dflash_mlx/engine/target_qwen_gdn.py:774-778
 *                             greedy_tokens_with_mask  dflash_mlx/engine/sampling.py:47-55
 *                             match_acceptance_length  dflash_mlx/engine/acceptance.py:9-16
 *                             (composed at dflash_mlx/engine/spec_epoch.py:2067-2072,2129)
 */
#ifndef DFLASH_B200_H_
#define DFLASH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
  DFL_OK = 0,
  DFL_ERR_NULL_POINTER = 1,  /* a required pointer is NULL */
  DFL_ERR_BAD_SHAPE = 2,     /* a size is out of the supported range */
  DFL_ERR_MISALIGNED = 3,    /* a pointer or row stride breaks an alignment rule */
  DFL_ERR_WORKSPACE = 4,     /* workspace missing or too small */
  DFL_ERR_CUDA = 5,          /* a CUDA runtime / driver call failed */
  DFL_ERR_UNSUPPORTED = 6    /* no sm_100 device, or an unsupported option */
};

/* Human-readable text for a status code (static storage). */
const char* dfl_status_string(int status);

/* Library version string (static storage). */
const char* dfl_version(void);

/* Reads and clears the device error word written by kernels on the current
 * device (bounded-wait time-outs, bad geometry).  Synchronises the device.
 * Returns DFL_OK and stores the word (0 = no error) in *device_error. */
int dfl_get_device_error(int* device_error);

/* ------------------------------------------------------------------------
 * Dense int4 (affine, group size 64) verify qmm:  y = x @ dequant(W)^T.
 *
 *   x       bf16 [M, K], row-major, 16-byte aligned
 *   w_q     uint32 [N, K/8], nibble i of word p = column 8p+i (low first), 16-byte aligned
 *   scales  bf16 [N, K/64];  biases bf16 [N, K/64]  (w = nib * scale + bias)
 *   y       bf16 [M, N], row-major
 * Constraints: 1 <= M <= 32, K % 64 == 0, K >= 64, 1 <= N <= 2097152.
 * workspace: at least dfl_verify_qmm_workspace_bytes(M, K, N) bytes of
 * device memory, 16-byte aligned.  Its first 64 KB hold split-K tile
 * counters that must be zero before the first call (zero-fill the buffer
 * once); every call leaves them zero again, so one buffer serves any
 * sequence of calls in stream order.  The rest is fp32 partial sums.  One
 * workspace must not be shared by calls that may run concurrently.
 * Replaces verify_matmul (dflash_mlx/verify_qmm.py:905-1022) and the
 * VerifyQuantizedLinear dispatch closure (dflash_mlx/verify_linear.py:118-309).
 * ---------------------------------------------------------------------- */
int dfl_verify_qmm_w4g64(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                         const uint16_t* biases, uint16_t* y, void* workspace,
                         size_t workspace_bytes, int M, int K, int N, void* stream);

/* Workspace bytes dfl_verify_qmm_w4g64 needs for this shape on the current
 * device; 0 with *status != DFL_OK on error. */
size_t dfl_verify_qmm_workspace_bytes(int M, int K, int N, int* status);

#ifdef __cplusplus
}
#endif

#endif /* DFLASH_B200_H_ */
