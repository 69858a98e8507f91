"""dflash-b200: the dflash-mlx target-verify hot path, B200-native.

Public surface (mirrors the reference's names):

* ``verify_matmul``, ``is_enabled``                      (dflash_mlx/verify_qmm.py)
* ``QuantizedLinear``, ``VerifyQuantizedLinear``, ``is_verify_eligible``,
  ``install_verify_linears``, ``prewarm_verify_kernels`` (dflash_mlx/verify_linear.py)

Every op runs hand-written sm_100a CUDA from ``libdflash_b200.so`` through
its C ABI (``include/dflash_b200.h``); there is no CPU fallback.
"""

from .verify_qmm import is_enabled, verify_matmul, qmm_w4g64
from .verify_linear import (
    QuantizedLinear,
    VerifyQuantizedLinear,
    install_verify_linears,
    is_verify_eligible,
    prewarm_verify_kernels,
)

__all__ = [
    "is_enabled",
    "verify_matmul",
    "qmm_w4g64",
    "QuantizedLinear",
    "VerifyQuantizedLinear",
    "install_verify_linears",
    "is_verify_eligible",
    "prewarm_verify_kernels",
]
