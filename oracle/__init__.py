"""CPU oracle for the dflash-mlx target-verify hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module: only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
/ ``--impl reference`` legs of ``bench.py`` use it, and only as the checker
(or as the timed CPU restatement of the reference), never as a fallback.

Each function restates the reference algorithm in NumPy and cites the
reference file:line it follows (paths relative to the dflash-mlx project):

* ``qmm``      -- ``dflash_mlx/verify_qmm.py:243-250`` (affine int4 dequant,
  ``w = float(nib) * s + b`` rounded to the activation dtype) and the stock
  ``mx.quantized_matmul(transpose=True)`` semantics exercised by
  ``tests/test_verify_qmm_parity.py:44-72``.
* ``moe``      -- the routed-expert ``gather_qmm`` path of mlx-lm's
  ``SwitchGLU`` (third party: mlx-lm >= 0.31.0, not vendored in the
  reference) as reached from ``dflash_mlx/engine/target_qwen_gdn.py:863-865``.
* ``lmhead``   -- ``engine/sampling.py:47-55`` (argmax with a -1e9 floor on
  suppressed ids) and ``engine/acceptance.py:9-16`` (sum of cumprod of
  matches), composed as at ``engine/spec_epoch.py:2067-2072``.
* ``gdn``      -- ``dflash_mlx/kernels.py:125-167`` (gated-delta forward with
  innovation tape), ``kernels.py:421-458`` (tree forward, used to pin the
  replay identity) and ``kernels.py:790-820`` (tape replay).

Parity pins (see ``tests/test_oracle_pins.py``):

* acceptance: the golden table of ``tests/test_engine_acceptance.py:11-24``;
* tape replay: the replay-equals-tree-state identity of
  ``tests/test_gated_delta_tree_kernel.py:162-178`` on the arange inputs of
  ``tests/test_gated_delta_tree_kernel.py:22-54``;
* qmm / MoE: no golden vectors exist in the reference (its tests compare
  against MLX at run time, and MLX cannot run on this machine).  The qmm
  oracle is pinned by hand-computed known-answer tests of the nibble layout
  only; MLX-relative parity is **unpinned**.
"""
