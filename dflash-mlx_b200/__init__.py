"""dflash-b200: the dflash-mlx target-verify hot path, B200-native.

Public surface (mirrors the reference's names):

* ``verify_matmul``, ``is_enabled``                      (dflash_mlx/verify_qmm.py)
* ``QuantizedLinear``, ``VerifyQuantizedLinear``, ``is_verify_eligible``,
  ``install_verify_linears``, ``prewarm_verify_kernels`` (dflash_mlx/verify_linear.py)
* ``tape_replay_kernel`` (dflash_mlx/kernels.py), ``RecurrentRollbackCache``
  (dflash_mlx/recurrent_rollback_cache.py), ``restore_after_acceptance``
  (dflash_mlx/engine/target_qwen_gdn.py)

Every op runs hand-written sm_100a CUDA from ``libdflash_b200.so`` through
its C ABI (``include/dflash_b200.h``); there is no CPU fallback.
"""

from . import checkpoint, kernels, lm_head, moe, qmm_plan
from .lm_head import lm_head_argmax_keys, lm_head_verify, match_acceptance_length, verify_accept
from .kernels import (gated_delta_kernel_with_tape, gated_delta_tree_kernel,
                      gated_delta_tree_tape_kernel, tape_replay_, tape_replay_kernel,
                      tree_depthwise_conv1d)
from .recurrent_rollback_cache import (
    RecurrentRollbackCache,
    arm_rollback,
    cleanup_generation_caches,
    clear_rollback_state,
    restore_after_acceptance,
)
from .verify_qmm import (is_enabled, verify_matmul, qmm_w4g64, repack_pairs, interleave_gate_up,
                         gate_up_silu)
from .qmm_plan import PlanPhase, ProjectionPlan, TiledWeight, qmm_tiled, tile_weight
from .verify_linear import (
    QuantizedLinear,
    VerifyQuantizedLinear,
    install_verify_linears,
    is_verify_eligible,
    prewarm_verify_kernels,
)

__all__ = [
    "gated_delta_tree_kernel",
    "gated_delta_tree_tape_kernel",
    "tree_depthwise_conv1d",
    "checkpoint",
    "lm_head_argmax_keys",
    "lm_head_verify",
    "match_acceptance_length",
    "verify_accept",
    "tape_replay_kernel",
    "tape_replay_",
    "RecurrentRollbackCache",
    "restore_after_acceptance",
    "is_enabled",
    "verify_matmul",
    "qmm_w4g64",
    "repack_pairs",
    "interleave_gate_up",
    "gate_up_silu",
    "qmm_plan",
    "PlanPhase",
    "ProjectionPlan",
    "TiledWeight",
    "qmm_tiled",
    "tile_weight",
    "QuantizedLinear",
    "VerifyQuantizedLinear",
    "install_verify_linears",
    "is_verify_eligible",
    "prewarm_verify_kernels",
]
