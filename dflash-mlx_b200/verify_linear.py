"""Drop-in verify linears for PyTorch modules.

Mirrors ``dflash_mlx/verify_linear.py``:

* ``QuantizedLinear``          -- the attribute layout of ``mlx.nn.QuantizedLinear``
  (``weight`` uint32 ``[N, K/8]``, ``scales``, ``biases``, optional ``bias``,
  ``group_size``, ``bits``, ``mode``) as a torch module, so models built for
  the MLX layout can be held on a B200;
* ``is_verify_eligible``       -- ``verify_linear.py:54-87`` (same env knobs
  ``DFLASH_VERIFY_MAX_N`` / ``DFLASH_VERIFY_INCLUDE``, read by ``settings.py``,
  and path tags);
* ``VerifyQuantizedLinear``    -- ``verify_linear.py:89-116``; every row count
  goes through the sm_100a qmm (the reference special-cases M=16 and M=4 and
  sends the rest to stock ``mx.quantized_matmul``);
* ``prewarm_verify_kernels``   -- ``verify_linear.py:311-336``;
* ``install_verify_linears``   -- ``verify_linear.py:338-361``.

Eligibility is narrower than the reference's because only the int4 g64
affine layout has a B200 kernel (bits 8 and group sizes 32/128 are not
implemented); ineligible modules are left in place, as in the reference.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
from torch import nn

from . import settings as _settings
from .verify_qmm import verify_matmul

_PROJ_TAGS = {
    "mlp.gate_proj": "mlp_gate",
    "mlp.up_proj": "mlp_up",
    "mlp.down_proj": "mlp_down",
    "self_attn.q_proj": "attn_q",
    "self_attn.k_proj": "attn_k",
    "self_attn.v_proj": "attn_v",
    "self_attn.o_proj": "attn_o",
    "linear_attn.in_proj_qkv": "gdn_qkv",
    "linear_attn.in_proj_z": "gdn_z",
    "linear_attn.out_proj": "gdn_o",
}


def _path_tag(path: str) -> str:
    for suffix, tag in _PROJ_TAGS.items():
        if path.endswith(suffix):
            return tag
    return "other"


class QuantizedLinear(nn.Module):
    """Affine-quantized linear with MLX's parameter layout, held in torch."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 bias: Optional[torch.Tensor] = None, *, group_size: int = 64, bits: int = 4,
                 mode: str = "affine"):
        super().__init__()
        self.group_size = int(group_size)
        self.bits = int(bits)
        self.mode = mode
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.bias = None

    @property
    def in_features(self) -> int:
        return int(self.weight.shape[1]) * (32 // self.bits)

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[0])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = verify_matmul(x, self.weight, self.scales, self.biases, transpose=True,
                          group_size=self.group_size, bits=self.bits)
        if self.bias is not None:
            y = y + self.bias
        return y


def is_verify_eligible(ql, path: str = "") -> bool:
    if not isinstance(ql, QuantizedLinear):
        return False
    if getattr(ql, "bits", None) != 4:
        return False
    if getattr(ql, "group_size", None) != 64:
        return False
    if getattr(ql, "mode", "affine") != "affine":
        return False
    n = int(ql.weight.shape[0])
    k = int(ql.weight.shape[1]) * (32 // ql.bits)
    if k % 64 != 0:
        return False
    cfg = _settings.read()
    if n >= cfg.max_n:
        return False
    return cfg.allows(_path_tag(path))


class VerifyQuantizedLinear(QuantizedLinear):
    """Verify-path wrapper; shares the wrapped module's tensors (no copy).

    ``enable_qmm`` (default: ``DFLASH_VERIFY_QMM == "1"``) is accepted and
    stored as ``enable_qmm`` for callers that inspect it.  In the reference it
    chooses between its Metal verify kernels and stock MLX; here every call
    runs the sm_100a kernel whatever its value, because there is no second
    implementation to choose (no CPU or library fallback).
    """

    @classmethod
    def from_quantized(cls, ql: QuantizedLinear, *,
                       enable_qmm: Optional[bool] = None) -> "VerifyQuantizedLinear":
        obj = cls(ql.weight.contiguous(), ql.scales.contiguous(), ql.biases.contiguous(),
                  getattr(ql, "bias", None), group_size=ql.group_size, bits=ql.bits,
                  mode=getattr(ql, "mode", "affine"))
        obj.enable_qmm = _settings.read().qmm if enable_qmm is None else bool(enable_qmm)
        obj.requires_grad_(False)
        return obj


def prewarm_verify_kernels(model: nn.Module, *, input_dtype=torch.bfloat16) -> int:
    """Run each distinct verify shape once at M=16 and M=4 (``verify_linear.py:311-336``)."""
    seen = set()
    warmed = 0
    for _, m in model.named_modules():
        if not isinstance(m, VerifyQuantizedLinear):
            continue
        k = m.in_features
        n = m.out_features
        key = (k, n, m.bits, m.group_size)
        if key in seen:
            continue
        seen.add(key)
        for rows in (16, 4):
            dummy = torch.zeros((1, rows, k), dtype=input_dtype, device=m.weight.device)
            m(dummy)
            warmed += 1
    return warmed


def install_verify_linears(model: nn.Module, *,
                           predicate: Optional[Callable[[str, QuantizedLinear], bool]] = None,
                           enable_qmm: Optional[bool] = None) -> int:
    """Swap every eligible ``QuantizedLinear`` for a ``VerifyQuantizedLinear``.

    Returns the number of modules swapped (``verify_linear.py:338-361``).
    """
    if predicate is None:
        predicate = lambda path, m: is_verify_eligible(m, path=path)  # noqa: E731
    swaps = []
    for path, mod in model.named_modules():
        if isinstance(mod, VerifyQuantizedLinear):
            continue
        if isinstance(mod, QuantizedLinear) and predicate(path, mod):
            swaps.append(path)
    for path in swaps:
        parent = model
        parts = path.split(".") if path else []
        for p in parts[:-1]:
            parent = getattr(parent, p)
        old = getattr(parent, parts[-1]) if parts else model
        new = VerifyQuantizedLinear.from_quantized(old, enable_qmm=enable_qmm)
        if parts:
            setattr(parent, parts[-1], new)
    return len(swaps)
