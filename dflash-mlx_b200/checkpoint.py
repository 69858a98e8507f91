"""MLX safetensors checkpoints of affine-quantized models -> this package's
``QuantizedLinear`` modules and the fused verify-layer weights.

The reference loads its target with ``mlx_lm.utils.load``
(``dflash_mlx/runtime/loading.py:175-213``) and then swaps eligible
``nn.QuantizedLinear`` modules for verify linears
(``verify_linear.py:338-361``).  The checkpoint it reads is a directory with

* ``config.json`` whose ``"quantization"`` (or ``"quantization_config"``)
  entry holds the default ``group_size`` / ``bits`` (and optionally ``mode``)
  plus per-module overrides keyed by module path (a dict, or ``false`` for a
  module left unquantized);
* one or more ``*.safetensors`` files, mapped by
  ``model.safetensors.index.json`` (``"weight_map": {tensor: file}``) when
  there are several.

Each quantized linear at module path ``p`` stores ``p.weight`` (uint32
``[N, K * bits / 32]``, low nibble first), ``p.scales`` and ``p.biases``
(``[N, K / group_size]`` in the model dtype) and optionally ``p.bias``.

The safetensors container is read here directly: an 8-byte little-endian
header length, a JSON header ``{name: {"dtype", "shape", "data_offsets":
[begin, end]}, "__metadata__": {...}}``, then the raw little-endian tensor
bytes, offsets counted from the end of the header.  Tensors are memory-mapped
and copied to the device one at a time.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Dict, Iterable, Optional, Tuple

import numpy as np
import torch

from .moe import QuantWeight
from .verify_linear import QuantizedLinear

# safetensors dtype tag -> (numpy storage dtype, torch dtype viewed from it)
_DTYPES = {
    "U32": (np.uint32, torch.int32),
    "I32": (np.int32, torch.int32),
    "BF16": (np.uint16, torch.bfloat16),
    "F16": (np.uint16, torch.float16),
    "F32": (np.float32, torch.float32),
    "U8": (np.uint8, torch.uint8),
    "I64": (np.int64, torch.int64),
}


def read_safetensors_header(path: Path) -> Tuple[dict, int]:
    """(header dict, byte offset of the data section) of one safetensors file."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        (n,) = struct.unpack("<Q", raw)
        if n > 100 << 20:
            raise ValueError(f"{path}: header length {n} is implausible")
        header = json.loads(f.read(n).decode("utf-8"))
    return header, 8 + n


@dataclass
class TensorRef:
    file: Path
    dtype: str
    shape: Tuple[int, ...]
    begin: int  # absolute byte offsets in the file
    end: int

    def numpy(self) -> np.ndarray:
        """The tensor as a read-only memory map (bf16 / fp16 as uint16 bits)."""
        if self.dtype not in _DTYPES:
            raise NotImplementedError(f"safetensors dtype {self.dtype} is not supported")
        npdt = np.dtype(_DTYPES[self.dtype][0]).newbyteorder("<")
        count = int(np.prod(self.shape)) if self.shape else 1
        if self.end - self.begin != count * npdt.itemsize:
            raise ValueError(f"{self.file}: tensor size does not match its shape {self.shape}")
        arr = np.memmap(self.file, dtype=npdt, mode="r", offset=self.begin, shape=(count,))
        return arr.reshape(self.shape)

    def torch(self, device) -> torch.Tensor:
        src = self.numpy()
        a = np.ascontiguousarray(src).astype(src.dtype.newbyteorder("="), copy=False)
        signed = {1: np.uint8, 2: np.int16, 4: np.int32, 8: np.int64}[a.itemsize]
        if a.dtype.kind != "f":
            a = a.view(signed)
        t = torch.from_numpy(np.array(a, copy=True))
        _, tdt = _DTYPES[self.dtype]
        return (t.view(tdt) if t.dtype != tdt else t).to(device)


class Checkpoint:
    """Tensor index and quantization config of an MLX checkpoint directory."""

    def __init__(self, path):
        self.path = Path(path)
        cfg_file = self.path / "config.json"
        self.config = json.loads(cfg_file.read_text()) if cfg_file.exists() else {}
        index = self.path / "model.safetensors.index.json"
        if index.exists():
            files = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        else:
            files = sorted(p.name for p in self.path.glob("*.safetensors"))
        if not files:
            raise FileNotFoundError(f"no safetensors files in {self.path}")
        self.tensors: Dict[str, TensorRef] = {}
        for name in files:
            f = self.path / name
            header, data0 = read_safetensors_header(f)
            for key, meta in header.items():
                if key == "__metadata__":
                    continue
                b, e = meta["data_offsets"]
                self.tensors[key] = TensorRef(f, meta["dtype"], tuple(meta["shape"]), data0 + b, data0 + e)
        q = self.config.get("quantization", self.config.get("quantization_config"))
        self.quantization = q if isinstance(q, dict) else {}

    def quant_spec(self, module_path: str) -> Optional[dict]:
        """{"group_size", "bits", "mode"} of a module, or None if unquantized."""
        q = self.quantization
        if not q:
            return None
        over = q.get(module_path)
        if over is False:
            return None
        base = {"group_size": int(q.get("group_size", 64)), "bits": int(q.get("bits", 4)),
                "mode": q.get("mode", "affine")}
        if isinstance(over, dict):
            base.update({k: over[k] for k in ("group_size", "bits", "mode") if k in over})
        return base

    def quantized_linear_paths(self) -> list:
        """Module paths with a uint32 weight plus scales (and biases)."""
        out = []
        for key, ref in self.tensors.items():
            if not key.endswith(".weight") or ref.dtype != "U32":
                continue
            p = key[: -len(".weight")]
            if p + ".scales" in self.tensors:
                out.append(p)
        return sorted(out)


def load_quantized_linears(path, device, *,
                           predicate: Optional[Callable[[str], bool]] = None) -> Dict[str, QuantizedLinear]:
    """Every quantized linear of the checkpoint (optionally filtered by module
    path) as a ``QuantizedLinear`` on ``device`` with the MLX tensors as is."""
    ck = Checkpoint(path)
    out: Dict[str, QuantizedLinear] = {}
    for p in ck.quantized_linear_paths():
        if predicate is not None and not predicate(p):
            continue
        spec = ck.quant_spec(p) or {"group_size": 64, "bits": 4, "mode": "affine"}
        w = ck.tensors[p + ".weight"].torch(device)
        s = ck.tensors[p + ".scales"].torch(device)
        b_ref = ck.tensors.get(p + ".biases")
        if b_ref is None:
            raise NotImplementedError(f"{p}: quantization without biases (mode {spec['mode']}) "
                                      "is not an affine int4 layer")
        b = b_ref.torch(device)
        bias = ck.tensors[p + ".bias"].torch(device) if p + ".bias" in ck.tensors else None
        k = w.shape[1] * 32 // spec["bits"]
        if s.shape != (w.shape[0], k // spec["group_size"]):
            raise ValueError(f"{p}: scales {tuple(s.shape)} do not match weight {tuple(w.shape)} "
                             f"at group_size {spec['group_size']}, bits {spec['bits']}")
        out[p] = QuantizedLinear(w, s, b, bias, group_size=spec["group_size"], bits=spec["bits"],
                                 mode=spec["mode"])
    return out


def fuse_rows(mods: Iterable[QuantizedLinear]) -> QuantWeight:
    """Projections that read the same input, concatenated along N (one launch)."""
    mods = list(mods)
    _check_fusable(mods)
    return QuantWeight(torch.cat([m.weight for m in mods]).contiguous(),
                       torch.cat([m.scales for m in mods]).contiguous(),
                       torch.cat([m.biases for m in mods]).contiguous())


def fuse_gate_up(gate: QuantizedLinear, up: QuantizedLinear) -> QuantWeight:
    """An MLP's gate and up projections interleaved in 16-row blocks, the
    layout of the fused gate|up + SiLU launch (``gate_up_silu``)."""
    from .verify_qmm import interleave_gate_up

    _check_fusable([gate, up])
    return QuantWeight(interleave_gate_up(gate.weight, up.weight).contiguous(),
                       interleave_gate_up(gate.scales, up.scales).contiguous(),
                       interleave_gate_up(gate.biases, up.biases).contiguous())


def pair_pack(qw: QuantWeight) -> QuantWeight:
    """The same weight with its nibbles in the pair-packed order (on the GPU)."""
    from .verify_qmm import repack_pairs

    return QuantWeight(repack_pairs(qw.q), qw.s, qw.b)


def _check_fusable(mods):
    if not mods:
        raise ValueError("nothing to fuse")
    k = mods[0].in_features
    for m in mods:
        if (m.bits, m.group_size, getattr(m, "mode", "affine")) != (4, 64, "affine"):
            raise NotImplementedError("only affine int4 group-64 projections are fused")
        if m.in_features != k:
            raise ValueError("fused projections must share the input width")
        if m.bias is not None:
            raise NotImplementedError("fused projections with an additive bias are not supported")
