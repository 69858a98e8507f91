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
 *   dfl_gdn_forward_tape   <- gated_delta_kernel_with_tape dflash_mlx/kernels.py:169-219
 *   dfl_gdn_tree_forward   <- gated_delta_tree_kernel / gated_delta_tree_tape_kernel
 *                                                      dflash_mlx/kernels.py:501-586
 *   dfl_tree_depthwise_conv1d <- tree_depthwise_conv1d dflash_mlx/kernels.py:647-688
 *   dfl_lmhead_argmax + dfl_lmhead_accept
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
  DFL_ERR_UNSUPPORTED = 6,   /* no sm_100 device, or an unsupported option */
  DFL_ERR_SCRATCH_LIMIT = 7  /* needs more scratch than the fixed no-allocation array */
};

/* Human-readable text for a status code (static storage). */
const char* dfl_status_string(int status);

/* Library version string (static storage). */
const char* dfl_version(void);

/* Reads and clears the device error word written by kernels on the current
 * device (bounded-wait time-outs, bad geometry).  Synchronises the device.
 * Returns DFL_OK and stores the word (0 = no error) in *device_error.  When
 * the word was set it also zero-fills the library's own no-allocation
 * scratch on that device (dfl_verify_qmm_w4g64_noalloc); caller workspaces
 * are the caller's to zero-fill. */
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
 * device memory, 16-byte aligned, zero before the first call (zero-fill it
 * once): it holds split-K partial sums whose words carry a validity bit,
 * and every call clears what it consumed, so one buffer serves any
 * sequence of calls in stream order.  After a call that reported a device
 * error (dfl_get_device_error) the buffer must be zero-filled again.  One
 * workspace must not be shared by calls that may run concurrently.
 * Replaces verify_matmul (dflash_mlx/verify_qmm.py:905-1022) and the
 * VerifyQuantizedLinear dispatch closure (dflash_mlx/verify_linear.py:118-309).
 * ---------------------------------------------------------------------- */
int dfl_verify_qmm_w4g64(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                         const uint16_t* biases, uint16_t* y, void* workspace,
                         size_t workspace_bytes, int M, int K, int N, void* stream);

/* The same contract with x, scales, biases and y all fp16 (the reference
 * builds a bf16 and an fp16 kernel per layer, dflash_mlx/verify_linear.py:
 * 163-164, and dispatches on x.dtype, verify_linear.py:241-247).  Uses the
 * same workspace size and the same workspace rules. */
int dfl_verify_qmm_w4g64_f16(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                             const uint16_t* biases, uint16_t* y, void* workspace,
                             size_t workspace_bytes, int M, int K, int N, void* stream);

/* Pair-packed weight order.  dfl_repack_w4_pairs rewrites MLX-packed int4
 * words so that nibble j of word p holds column 8p + 2j and nibble 4 + j
 * column 8p + 2j + 1 (j = 0..3); dst may equal src (each word maps to
 * itself).  n_words % 4 == 0, both pointers 16-byte aligned.  A load-time
 * layout of this library, not a reference format: the reference keeps MLX
 * order and its kernels take that layout directly (verify_qmm.py:905).
 * dfl_verify_qmm_w4g64_pairs / _pairs_f16 are dfl_verify_qmm_w4g64 / _f16
 * on repacked weights (same arguments, workspace and results up to fp32
 * summation order): the dequantiser then yields natural K order and x goes
 * to shared memory by TMA without a permutation step. */
int dfl_repack_w4_pairs(const uint32_t* src, uint32_t* dst, size_t n_words, void* stream);
int dfl_verify_qmm_w4g64_pairs(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                               const uint16_t* biases, uint16_t* y, void* workspace,
                               size_t workspace_bytes, int M, int K, int N, void* stream);
int dfl_verify_qmm_w4g64_pairs_f16(const uint16_t* x, const uint32_t* w_q,
                                   const uint16_t* scales, const uint16_t* biases, uint16_t* y,
                                   void* workspace, size_t workspace_bytes, int M, int K, int N,
                                   void* stream);

/* Gate/up projection pair with SiLU*up fused into the epilogue, on MLX-packed
 * (dfl_verify_qmm_w4g64_silu) or pair-packed (_pairs_silu, _pairs_silu_f16)
 * weights: w_q / scales / biases hold the gate and up rows
 * interleaved in blocks of 32 (rows 32b..32b+15 = gate rows 16b..16b+15,
 * rows 32b+16..32b+31 = up rows 16b..16b+15), N = 2 * intermediate,
 * N % 32 == 0.  h [M, N/2] = silu(gate) * up with gate and up each rounded
 * to the activation dtype first and the SiLU in fp32, exactly as
 * dfl_silu_mul_bf16 on the two projections.  Same workspace rules.
 * Replaces the MLP's gate_proj/up_proj pair and nn.silu(gate) * up of the
 * verify forward (mlx-lm's MLP, reached from the target model's layers at
 * dflash_mlx/engine/target_qwen_gdn.py:863-865). */
int dfl_verify_qmm_w4g64_silu(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                              const uint16_t* biases, uint16_t* h, void* workspace,
                              size_t workspace_bytes, int M, int K, int N, void* stream);
int dfl_verify_qmm_w4g64_pairs_silu(const uint16_t* x, const uint32_t* w_q,
                                    const uint16_t* scales, const uint16_t* biases, uint16_t* h,
                                    void* workspace, size_t workspace_bytes, int M, int K, int N,
                                    void* stream);
int dfl_verify_qmm_w4g64_pairs_silu_f16(const uint16_t* x, const uint32_t* w_q,
                                        const uint16_t* scales, const uint16_t* biases,
                                        uint16_t* h, void* workspace, size_t workspace_bytes,
                                        int M, int K, int N, void* stream);

/* The dense qmm's stream-K split of `total` (tile, K unit) pairs over `grid`
 * CTAs, as the launches use it: CTA c takes units [ubeg[c], ubeg[c + 1]),
 * ubeg has grid + 1 entries, the first half of the CTAs weigh 1 and the
 * weight falls linearly to 1 - skew / 256 at the last CTA (*skew_used, the
 * built-in skew clamped so every range keeps at least one unit).  Host-only
 * (no device access); exposed for tests of the split. */
int dfl_qmm_stream_k_ranges(int total, int grid, int* ubeg, int* skew_used);

/* Workspace bytes dfl_verify_qmm_w4g64 needs for this shape on the current
 * device; 0 with *status != DFL_OK on error.  No counterpart in the
 * reference (MLX allocates the split-K buffer of verify_qmm.py:993-1001
 * itself). */
size_t dfl_verify_qmm_workspace_bytes(int M, int K, int N, int* status);

/* dfl_verify_qmm_w4g64 without a workspace argument, for callers that cannot
 * allocate device memory.  No counterpart in the reference (MLX allocates
 * its own buffers).  Same x / w_q / scales / biases / y / shape rules and the
 * same results.  Split-K scratch is a fixed 8 MiB device array inside the
 * library, shared by every call on a device:
 *   - a shape whose dfl_verify_qmm_workspace_bytes exceeds 8 MiB returns
 *     DFL_ERR_SCRATCH_LIMIT (never for M <= 32: the need is at most 2.6 MB);
 *   - the first call on a device looks the array up on that device (make it
 *     before any stream capture there);
 *   - the first call on a device zero-fills the array on `stream`; every
 *     call leaves it zero again, so calls in stream order are safe; calls
 *     that can overlap in time race;
 *   - a call that timed out can leave partial sums behind; the next
 *     dfl_get_device_error on that device that finds the error word set
 *     zero-fills the array again, so check it before trusting later calls.
 * Allocates nothing. */
int dfl_verify_qmm_w4g64_noalloc(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                                 const uint16_t* biases, uint16_t* y, int M, int K, int N,
                                 void* stream);

/* ------------------------------------------------------------------------
 * Projection plans: one persistent launch for a sequence of int4 g64
 * verify projections (a decoder layer, or a whole layer stack).
 *
 * Weights first go through a load-time repack into the tiled layout:
 * dfl_w4_tiled_bytes(N, K) bytes (ceil(N/128) * ceil(K/512) blocks of
 * 36864 bytes: one contiguous block per 128 rows x 512 columns, nibbles in
 * the order the kernel's dequant threads read them, then that block's
 * scales and biases).  dfl_repack_w4_tiled reads MLX-packed w_q [N, K/8]
 * and bf16 scales / biases [N, K/64] (K % 64 == 0); rows and columns past
 * N / K are stored as zero weights.  subnormal = 1 stores every scale as
 * scale * 2^133 for the kernel's subnormal dequantiser and needs
 * |scale| < 2^-5 (finite) for every group; a scale outside that range is
 * stored as 0 and sets the device error word (kDevBadInput), so check the
 * scales first and pass subnormal = 0 for such a tensor.  Both forms give
 * the dequantised weights bit for bit (w = nib * scale + bias, rounded
 * once to bf16, as dflash_mlx/verify_qmm.py:249).  Not a reference format
 * (the reference keeps MLX order, verify_qmm.py:905); like concatenating
 * projections, it is done once per weight.
 *
 * A plan is an array of phases run in order.  Phase p computes
 * y = x @ dequant(W)^T for M <= 128 rows (bf16 x [M, K] with row stride ldx,
 * ldx % 8 == 0, x 16-byte aligned; y [M, N] with row stride ldy) or, with
 * DFL_PHASE_SILU, h [M, N/2] = silu(gate) * up over gate/up rows
 * interleaved in blocks of 16 (N % 32 == 0, as dfl_verify_qmm_w4g64_silu).
 * DFL_PHASE_SUBNORMAL must match the subnormal flag of the phase's repack.
 * dep = q (an earlier phase) makes the phase read x only after every output
 * of phase q is written (x may be phase q's y); dep = -1 reads x at once.
 * DFL_PHASE_GROUPED runs one projection per problem of a sorted route
 * table (dfl_moe_sort_pairs; route, read on the device when the plan runs):
 * w_tiled holds `experts` weights [N, K] (N % 128 == 0) tiled one after the
 * other, x and y have M <= 256 rows (the sorted rows), and problem i
 * multiplies its rows [route[1+2i], route[3+2i]) (at most problem_rows of
 * them; a plan with grouped phases runs at a 16- or 32-row token tile, so
 * problem_rows <= 32 and every dense phase of it has M <= 32) by expert
 * route[2+2i]'s weight.  With DFL_PHASE_SCATTER
 * (grouped only) output row r goes to row route[514 + r] of y instead of r.
 * Expert ids and rows outside the phase's bounds set the device error word
 * and read expert 0 / store nothing.
 * Results equal dfl_verify_qmm_w4g64 on the same weights up to fp32
 * summation order.  The plan's token tile (16, 32, 64 or 128 rows) follows
 * its largest M, and every phase runs at that tile, so all rows of a phase
 * share one read of its weights; more rows than 128 take one phase per
 * 128-row slice.  Each phase's split over the SMs depends only on its own
 * shape, so a phase gives the same bits in any plan with the same tile.
 *
 * dfl_qmm_plan_encode writes the plan for the current device into a host
 * buffer of dfl_qmm_plan_bytes(n_phases) bytes; copy those bytes to a
 * 64-byte-aligned device buffer (any stream-ordered copy) before the first
 * run.  The x / y / weight pointers are baked in: re-encode when they
 * change.  dfl_qmm_plan_run launches the plan (one cooperative launch of
 * one CTA per SM) with a workspace of dfl_qmm_plan_workspace_bytes bytes,
 * zero before the first run; every run leaves its first 64 KB (counters and
 * phase stamps) zero again, and the split-K area after it may keep data
 * that no later run reads before stamping it.  After a run that reported a
 * device error (dfl_get_device_error) zero the workspace again.  One
 * workspace must not be shared by runs that may overlap.  No counterpart in
 * the reference (it launches one Metal kernel per projection through
 * VerifyQuantizedLinear, dflash_mlx/verify_linear.py:266-286); it replaces
 * that sequence of calls for the verify rows of one or more requests.
 * ---------------------------------------------------------------------- */
#define DFL_PHASE_SILU 1
#define DFL_PHASE_SUBNORMAL 2
#define DFL_PHASE_GROUPED 4
#define DFL_PHASE_SCATTER 8

typedef struct dfl_qmm_phase {
  const void* x;        /* bf16 [M, K], row stride ldx elements */
  void* y;              /* bf16 [M, N] (SiLU: [M, N/2]), row stride ldy elements */
  const void* w_tiled;  /* dfl_repack_w4_tiled output for this [N, K] weight */
  int M, K, N;
  int ldx, ldy;
  int flags;            /* DFL_PHASE_SILU | DFL_PHASE_SUBNORMAL | DFL_PHASE_GROUPED | DFL_PHASE_SCATTER */
  int dep;              /* -1, or an earlier phase whose outputs x reads */
  const int32_t* route; /* DFL_PHASE_GROUPED: sorted route table (dfl_moe_sort_pairs), else NULL */
  int experts;          /* DFL_PHASE_GROUPED: experts stacked in w_tiled */
  int problem_rows;     /* DFL_PHASE_GROUPED: rows of the largest problem (tokens per expert) */
} dfl_qmm_phase;

size_t dfl_w4_tiled_bytes(int N, int K);
int dfl_repack_w4_tiled(const uint32_t* w_q, const uint16_t* scales, const uint16_t* biases,
                        int N, int K, int subnormal, void* dst, size_t dst_bytes, void* stream);
size_t dfl_qmm_plan_bytes(int n_phases);
int dfl_qmm_plan_encode(const dfl_qmm_phase* phases, int n_phases, void* plan_host,
                        size_t plan_bytes);
size_t dfl_qmm_plan_workspace_bytes(const void* plan_host, int* status);
int dfl_qmm_plan_run(const void* plan_host, const void* plan_dev, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Failure handling of plans.  Every wait inside a plan run is bounded
 * (1 s by default); when one runs out the run sets the device error word
 * (dfl_get_device_error), records where it gave up in the workspace and
 * every CTA winds down and exits: the launch ends, nothing hangs, and the
 * workspace must be zero-filled before the next run.
 * dfl_qmm_plan_last_timeout reads that record from a host copy of the
 * workspace's first 64 KB: role (1 dependency, 2 slot guard, 3 split-K
 * partial, 4 producer, 5 MMA, 6 dequant, 7 x-slot, 8 accumulator; 0 = none),
 * phase and CTA of the first wait that ran out.
 * dfl_qmm_plan_set_test_fault edits an encoded host plan for tests of that
 * path: skip_partial_cta (-1 = none) makes that CTA withhold its split-K
 * partials, so the CTA that sums them waits until wait_limit_ns (1 ms .. 1 s)
 * runs out (a wait on an earlier phase's completion counter runs twice the
 * limit, so the first-hand wait is the one recorded).  Re-encode the plan (or
 * set -1 and 1e9) to run normally again.
 * No counterpart in the reference (its Metal kernels have no waits). */
int dfl_qmm_plan_set_test_fault(void* plan_host, int skip_partial_cta, uint64_t wait_limit_ns);
int dfl_qmm_plan_last_timeout(const void* workspace_host_words, int* role, int* phase, int* cta);

/* ------------------------------------------------------------------------
 * GatedDeltaNet tape-replay rollback.
 *
 * For every sequence b, value head hv and replayed step t:
 *     S[dv, dk] <- S[dv, dk] * g_t  (g_t per head, or per dk when g_vectorized)
 *     S[dv, dk] <- S[dv, dk] + tape_t[dv] * k_t[dk]
 * each a separately rounded fp32 operation; k head hk = hv / (Hv / Hk).
 * Step t of sequence b is replayed when t < steps[b] (steps NULL: all T) and
 * mask[b, t] != 0 (mask NULL: all).  state_out may equal state_in (in place;
 * heads with no replayed step are then not touched).
 *   tape   fp32 [B, T, Hv, Dv]          k  [B, T, Hk, Dk], bf16 (k_is_bf16) or fp32
 *   g      fp32 [B, T, Hv] or [B, T, Hv, Dk]
 *   steps  int32 [B] or NULL            mask uint8 [B, T] or NULL
 *   state  fp32 [B, Hv, Dv, Dk], 16-byte aligned
 * Constraints: Dk in {32, 64, 128, 256}, Dv * Dk <= 16384, Hv % Hk == 0, T <= 64.
 * Replaces tape_replay_kernel (dflash_mlx/kernels.py:822-868) as called by
 * RecurrentRollbackCache.rollback (dflash_mlx/recurrent_rollback_cache.py:142-165).
 * ---------------------------------------------------------------------- */
int dfl_gdn_tape_replay(const float* tape, const void* k, int k_is_bf16, const float* g,
                        int g_vectorized, const int32_t* steps, const uint8_t* mask,
                        const float* state_in, float* state_out, int B, int T, int Hv, int Hk,
                        int Dv, int Dk, void* stream);

/* GatedDeltaNet verify forward that records the innovation tape.
 *
 * For every sequence b, value head hv (q/k head hk = hv / (Hv / Hk)) and step t
 * with mask[b, t] != 0 (mask NULL: all steps):
 *     S' = S * g_t;  kv = S' k_t;  delta = (v_t - kv) * beta_t;
 *     S = S' + delta (x) k_t;  y_t = S q_t;  tape_t = delta
 * (state updates separately rounded fp32, in tape-replay order, so replaying
 * the tape over the first a steps reproduces the state after a steps exactly).
 * A masked-out step leaves S and writes tape = 0, y = 0.
 *   q, k   bf16 [B, T, Hk, Dk]      v bf16 [B, T, Hv, Dv]
 *   g      fp32 [B, T, Hv] or [B, T, Hv, Dk] (g_vectorized)    beta fp32 [B, T, Hv]
 *   state  fp32 [B, Hv, Dv, Dk], 16-byte aligned (state_out may equal state_in)
 *   y      bf16 [B, T, Hv, Dv]      tape fp32 [B, T, Hv, Dv]
 * Constraints: Dk in {32, 64, 128, 256}, Dv % 32 == 0, Hv % Hk == 0, T <= 64.
 * Replaces gated_delta_kernel_with_tape (dflash_mlx/kernels.py:169-219; Metal
 * body :28-101; mx-op reference _gated_delta_ops_with_tape :125-167). */
int dfl_gdn_forward_tape(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                         int g_vectorized, const float* beta, const uint8_t* mask,
                         const float* state_in, float* state_out, uint16_t* y, float* tape,
                         int B, int T, int Hv, int Hk, int Dv, int Dk, void* stream);

/* ------------------------------------------------------------------------
 * DDTree verify: the GDN recurrence over a token tree.
 *
 * Node t starts from the state of node parent_ids[t] (parents before
 * children; -1 = state_in) and applies one gated delta step (the update of
 * dfl_gdn_forward_tape).  Writes y [B, T, Hv, Dv] (input dtype), every node's
 * state to node_states [B, T, Hv, Dv, Dk] (fp32) and, when tape != NULL,
 * delta to tape [B, T, Hv, Dv] (fp32).  q, k [B, T, Hk, Dk] and v are bf16
 * (inputs_f32 = 0) or fp32 (inputs_f32 = 1); g fp32 [B, T, Hv] or
 * [B, T, Hv, Dk] (g_vectorized); beta fp32 [B, T, Hv]; parent_ids int32 [T]
 * on the device.  A parent id outside [-1, t) is recorded in the device error
 * word and that node starts from state_in.
 * Constraints: Dk in {32, 64, 128, 256}, Dv % 4 == 0, Hv % Hk == 0, T <= 64.
 * Replaces gated_delta_tree_kernel (node_states = its tree_states) and
 * gated_delta_tree_tape_kernel (node_states as scratch)
 * (dflash_mlx/kernels.py:501-586; Metal bodies :222-420). */
int dfl_gdn_tree_forward(const void* q, const void* k, const void* v, const float* g,
                         int g_vectorized, const float* beta, const float* state_in,
                         const int32_t* parent_ids, void* y, float* node_states, float* tape,
                         int B, int T, int Hv, int Hk, int Dv, int Dk, int inputs_f32,
                         void* stream);

/* Depthwise causal conv1d along tree paths, then SiLU:
 *   out[b, t, c] = silu(sum_w x(path_indices[t, w]) * weight[c, w] (+ bias[c]))
 * where slot s < K-1 reads prefix[b, s, c] and slot s >= K-1 reads
 * qkv[b, s - (K-1), c]; fp32 accumulation in w order.  qkv / prefix / out are
 * bf16 (inputs_f32 = 0) or fp32; weight fp32 [C, K]; bias fp32 [C] or NULL;
 * path_indices int32 [T, K].  A slot outside [0, K-1+T) is recorded in the
 * device error word and reads 0.  Replaces tree_depthwise_conv1d
 * (dflash_mlx/kernels.py:647-688; Metal body :588-629). */
int dfl_tree_depthwise_conv1d(const void* qkv, const void* prefix, const float* weight,
                              const float* bias, const int32_t* path_indices, void* out, int B,
                              int T, int C, int K, int inputs_f32, void* stream);

/* ------------------------------------------------------------------------
 * lm_head verify epilogue.
 *
 * dfl_lmhead_argmax: for the R = B * T hidden rows h (bf16 [R, D]) and one
 * vocabulary shard w (bf16 [V, D], global ids v_begin .. v_begin + V - 1),
 * computes each row's bf16 logits h . w_v (fp32 accumulation, rounded to
 * bf16 like the reference's bf16 logits), replaces suppressed ids
 * (suppress[v_begin + v] != 0; suppress may be NULL) by the bf16 value of
 * -1e9, and writes one 64-bit key per row: high 32 bits an order-preserving
 * image of the winning logit, low 32 bits 0xFFFFFFFF - id.  The largest key
 * is the largest logit with ties to the lowest id (argmax's first index),
 * so keys of several shards combine with max.  Logits are never written.
 * Constraints: 1 <= R <= 4096, D % 8 == 0, h and w 16-byte aligned.
 * workspace: dfl_lmhead_workspace_bytes(R, D, V) bytes (64 KB of counters +
 * 8 bytes per row); the same convention as every workspace here: zero
 * before the first call, and every call leaves all of it zero again, so one
 * buffer serves any sequence of calls (qmm, MoE qmm, lm_head) in stream order.
 * Replaces logits_from_hidden (dflash_mlx/engine/target_qwen_gdn.py:774-778)
 * + greedy_tokens_with_mask (dflash_mlx/engine/sampling.py:47-55).
 * ---------------------------------------------------------------------- */
int dfl_lmhead_argmax(const uint16_t* h, const uint16_t* w, int R, int D, int V, int v_begin,
                      const uint8_t* suppress, uint64_t* keys, void* workspace,
                      size_t workspace_bytes, void* stream);

size_t dfl_lmhead_workspace_bytes(int R, int D, int V, int* status);

/* dfl_lmhead_accept: reduces the keys of G shards (keys [G][B*T]), writes the
 * posterior ids [B, T], and with verify_ids [B, T] (verify_ids[b, 0] the staged
 * token, verify_ids[b, 1:] the drafts) the acceptance length
 * sum_i prod_{j<=i} [verify_ids[b, j+1] == posterior[b, j]] (0 .. T-1) and the
 * next staged token posterior[b, acceptance].  verify_ids, acceptance,
 * next_token and max_logit (the winning bf16 logit as fp32) may be NULL.
 * Replaces match_acceptance_length (dflash_mlx/engine/acceptance.py:9-16) as
 * composed at dflash_mlx/engine/spec_epoch.py:2067-2072,2129. */
int dfl_lmhead_accept(const uint64_t* keys, int G, const int32_t* verify_ids, int B, int T,
                      int32_t* posterior, int32_t* acceptance, int32_t* next_token,
                      float* max_logit, void* stream);

/* dfl_match_acceptance: acceptance[b] = length of the common prefix of
 * drafted[b, :L] and posterior[b, :L] (int32 [B, L] each).
 * Replaces match_acceptance_length (dflash_mlx/engine/acceptance.py:9-16). */
int dfl_match_acceptance(const int32_t* drafted, const int32_t* posterior, int B, int L,
                         int32_t* acceptance, void* stream);

/* ------------------------------------------------------------------------
 * MoE expert path (routed experts of one verify block).
 *
 * dfl_moe_route: router logits fp32 [T, E] (T <= 16 tokens) -> top_k experts
 * per token (largest logit first, ties to the lower id), their softmax
 * weights renormalised over the k kept experts (fp32 [T, top_k]), expert ids
 * (int32 [T, top_k]) and a route table of dfl_moe_route_table_ints(E) int32:
 * [0] number P of active experts, [1..E] their ids (ascending), [1+E..]
 * rows per active expert, then per active expert 16 token rows and 16 pair
 * rows (pair = t * top_k + j).  Everything stays on the device.
 *
 * dfl_moe_qmm_w4g64: for every active expert e (P read from the route table
 * on the device), y[pair rows] = x[rows] @ dequant(W_e)^T with W as for
 * dfl_verify_qmm_w4g64 but stacked per expert: w_q uint32 [E, N, K/8],
 * scales / biases bf16 [E, N, K/64].  x rows are the table's token rows
 * (gather_by_pair = 0; x is [T, K]) or its pair rows (gather_by_pair = 1; x is
 * [T * top_k, K]); y is [T * top_k, N].  Each active expert's weights are read
 * once.  max_problems bounds P (grid size); workspace as for the dense qmm
 * with dfl_moe_qmm_workspace_bytes.  gather_by_pair bit 1 (value 2) states
 * that the route table was complete before the previous launch on the stream
 * started (e.g. two launches back, with plain stream order before that):
 * the kernel then streams weights before the previous launch finishes, like
 * the dense qmm.
 *
 * dfl_silu_mul_bf16: out = bf16(silu(gate) * up), fp32 math.
 * dfl_moe_combine: y[t] = bf16(sum_j weights[t, j] * pair_out[t * top_k + j]
 * (+ shared[t])), fp32 in slot order.
 *
 * Replaces the mlx-lm SwitchGLU -> mx.gather_qmm expert block (third party,
 * not in the reference tree) that the reference reaches from the decoder
 * layers at dflash_mlx/engine/target_qwen_gdn.py:863-865.
 * ---------------------------------------------------------------------- */
int dfl_moe_route(const float* logits, int T, int E, int top_k, int32_t* route_table,
                  float* weights, int32_t* topk_ids, void* stream);
size_t dfl_moe_route_table_ints(int E);
int dfl_moe_qmm_w4g64(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                      const uint16_t* biases, uint16_t* y, const int32_t* route,
                      int gather_by_pair, int max_problems, int E, int K, int N, void* workspace,
                      size_t workspace_bytes, void* stream);
size_t dfl_moe_qmm_workspace_bytes(int max_problems, int K, int N, int* status);
/* The grouped qmm over each expert's gate/up pair interleaved in blocks of
 * 32 rows (as dfl_verify_qmm_w4g64_pairs_silu; N = 2 * intermediate,
 * N % 32 == 0) with SiLU*up fused into the epilogue: h [rows_out, N/2]. */
int dfl_moe_qmm_w4g64_silu(const uint16_t* x, const uint32_t* w_q, const uint16_t* scales,
                           const uint16_t* biases, uint16_t* h, const int32_t* route,
                           int gather_by_pair, int max_problems, int E, int K, int N,
                           void* workspace, size_t workspace_bytes, void* stream);
int dfl_silu_mul_bf16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int n,
                      void* stream);

/* dfl_silu_mul_rows_bf16: out[r, c] = bf16(silu(gate[r * ld + c]) * up[r * ld + c])
 * for r < rows, c < cols (out contiguous [rows, cols], ld >= cols): the SiLU
 * gate of a fused gate|up projection output read in place.  Same math as
 * dfl_silu_mul_bf16 (mlx-lm SwitchGLU / dense MLP activation). */
int dfl_silu_mul_rows_bf16(const uint16_t* gate, const uint16_t* up, int ld, uint16_t* out,
                           int rows, int cols, void* stream);
int dfl_moe_combine(const uint16_t* pair_out, const float* weights, const uint16_t* shared,
                    uint16_t* y, int T, int top_k, int H, void* stream);

/* Sorted route table for grouped plan phases (DFL_PHASE_GROUPED).
 * dfl_moe_sort_pairs orders the T * top_k (token, slot) pairs of topk_ids
 * (int32 [T, top_k], ids in [0, E); T * top_k <= 256) by expert id, then by
 * pair index (token, then slot), and writes, on the device:
 *   route (dfl_moe_sorted_route_ints() int32): [0] number P of active
 *     experts; [1 + 2i] first sorted row of problem i for i <= P
 *     ([1 + 2P] = T * top_k); [2 + 2i] expert of problem i (ascending);
 *     [514 + r] pair row (t * top_k + j) of sorted row r;
 *   x_sorted bf16 [T * top_k, H]: row r = x[pair row r / top_k];
 *   x_copy (optional, NULL to skip) bf16 [T, H] = x, the input buffer of a
 *     plan's dense phases (the shared expert), filled by the same launch.
 * x is bf16 [T, H] with row stride ldx (H % 8 == 0, ldx % 8 == 0, 16-byte
 * aligned).  An id outside [0, E) sets the device error word and the table
 * gets P = 0.  The grouped gate/up phase reads x_sorted and writes its rows
 * in sorted order; the grouped down phase (DFL_PHASE_SCATTER) writes row r
 * to pair row route[514 + r], so pair_out is ready for dfl_moe_combine.
 * Replaces the gather/sort inside mlx-lm's SwitchGLU -> mx.gather_qmm
 * (sort_indices; third party), reached from
 * dflash_mlx/engine/target_qwen_gdn.py:863-865. */
size_t dfl_moe_sorted_route_ints(void);
int dfl_moe_sort_pairs(const int32_t* topk_ids, int T, int top_k, int E, const uint16_t* x,
                       int ldx, int H, int32_t* route, uint16_t* x_sorted, uint16_t* x_copy,
                       void* stream);
/* dfl_moe_route_sorted: dfl_moe_route's top-k ids and weights (same values
 * bit for bit; T <= 16, E <= 4096) and dfl_moe_sort_pairs' table, sorted rows
 * and x copy, in one launch (no dfl_moe_route table).  shared_expert = 1
 * appends one more problem, expert E (a shared expert stacked after the E
 * routed ones), whose rows are the T tokens: sorted rows T * top_k + t =
 * x[t], mapped to pair rows T * top_k + t (x_sorted then has T * top_k + T
 * rows, at most 256), so a layer's shared expert runs in the same grouped
 * phases as its routed experts.  A token whose top-k finds no finite logit
 * sets the device error word and the table gets P = 0. */
int dfl_moe_route_sorted(const float* logits, int T, int E, int top_k, int shared_expert,
                         const uint16_t* x, int ldx, int H, int32_t* route, float* weights,
                         int32_t* topk_ids, uint16_t* x_sorted, uint16_t* x_copy, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DFLASH_B200_H_ */
