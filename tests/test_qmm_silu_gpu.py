"""Fused gate/up projection + SiLU*up epilogue (``gate_up_silu``).

The MLP's gate and up weights are interleaved in blocks of 16 rows and
pair-packed once at load; one launch then writes h = silu(gate) * up.
Checks: (1) bit-identical to the unfused path on the same weights (the same
kernel writing both projections, then the SiLU*up kernel); (2) against the
CPU oracle on the separate gate and up weights (each projection rounded to
the activation dtype, SiLU in fp32), |h - ref| <= 1e-2 + 2e-2 |ref|;
(3) fp16 activations; (4) the row-count rule (N % 32 == 0).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import bf16_to_np_bits, to_dev_bf16, to_dev_u32
from oracle import bf16 as obf16
from oracle import moe as omoe
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu


def _fused(pkg, dev, wg, sg, bg, wu, su, bu, to16):
    import torch

    w = pkg.interleave_gate_up(to_dev_u32(wg, dev), to_dev_u32(wu, dev))
    s = pkg.interleave_gate_up(to16(sg, dev), to16(su, dev))
    b = pkg.interleave_gate_up(to16(bg, dev), to16(bu, dev))
    return pkg.repack_pairs(w.contiguous()), s.contiguous(), b.contiguous()


def _unfused(pkg, x, w, s, b):
    """Same weights through the plain qmm, then de-interleave and SiLU*up."""
    y = pkg.qmm_w4g64(x, w, s, b, layout="pairs")
    m, n = y.shape
    y4 = y.view(m, n // 32, 2, 16)
    gate = y4[:, :, 0, :].reshape(m, n // 2)
    up = y4[:, :, 1, :].reshape(m, n // 2)
    from dflash_mlx_b200.moe import silu_mul

    return silu_mul(gate.contiguous(), up.contiguous())


def _ref_h(x, wg, sg, bg, wu, su, bu, dtype="bf16"):
    g = oqmm.qmm(x, wg, sg, bg, accum=np.float32, dtype=dtype)
    u = oqmm.qmm(x, wu, su, bu, accum=np.float32, dtype=dtype)
    gf, uf = oqmm._to_f32(g, dtype), oqmm._to_f32(u, dtype)
    return oqmm._from_f32((omoe.silu(gf) * uf).astype(np.float32), dtype)


@pytest.mark.parametrize("M,K,I", [
    (16, 5120, 17408),   # the benchmark's MLP
    (1, 1600, 48),       # K % 512 != 0, ragged last tile
    (17, 1024, 80),      # MT = 32
    (32, 512, 4096),
])
def test_gate_up_silu_bf16(pkg, dev, M, K, I):
    rng = np.random.default_rng(M * 13 + K + I)
    wg, sg, bg = oqmm.synth_weights(rng, I, K)
    wu, su, bu = oqmm.synth_weights(rng, I, K)
    x = oqmm.synth_x(rng, M, K)
    w, s, b = _fused(pkg, dev, wg, sg, bg, wu, su, bu, to_dev_bf16)
    xd = to_dev_bf16(x, dev)
    h = pkg.gate_up_silu(xd, w, s, b)
    assert tuple(h.shape) == (M, I)
    hb = bf16_to_np_bits(h)
    assert np.array_equal(hb, bf16_to_np_bits(_unfused(pkg, xd, w, s, b)))
    ref = obf16.to_f32(_ref_h(x, wg, sg, bg, wu, su, bu)).astype(np.float64)
    got = obf16.to_f32(hb).astype(np.float64)
    bad = np.abs(got - ref) > 1e-2 + 2e-2 * np.abs(ref)
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} outside tolerance"


def test_gate_up_silu_f16(pkg, dev):
    import torch

    def to_dev_f16(a, d):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(d).view(torch.float16)

    rng = np.random.default_rng(77)
    M, K, I = 16, 2048, 1024
    wg, sg, bg = oqmm.synth_weights(rng, I, K, dtype="f16")
    wu, su, bu = oqmm.synth_weights(rng, I, K, dtype="f16")
    x = oqmm.synth_x(rng, M, K, dtype="f16")
    w, s, b = _fused(pkg, dev, wg, sg, bg, wu, su, bu, to_dev_f16)
    h = pkg.gate_up_silu(to_dev_f16(x, dev), w, s, b)
    assert h.dtype == torch.float16
    got = h.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = _ref_h(x, wg, sg, bg, wu, su, bu, dtype="f16")
    g64 = got.view(np.float16).astype(np.float64)
    r64 = ref.view(np.float16).astype(np.float64)
    bad = np.abs(g64 - r64) > 1e-2 + 2e-2 * np.abs(r64)
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} outside tolerance"


def test_gate_up_silu_rejects_rows_not_multiple_of_32(pkg, dev):
    import torch
    from dflash_mlx_b200 import _lib

    lib = _lib.load()
    x = torch.zeros((16, 512), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((48, 64), dtype=torch.int32, device=dev)
    s = torch.zeros((48, 8), dtype=torch.bfloat16, device=dev)
    h = torch.zeros((16, 24), dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(1 << 22, dtype=torch.uint8, device=dev)
    st = lib.dfl_verify_qmm_w4g64_pairs_silu(x.data_ptr(), w.data_ptr(), s.data_ptr(), s.data_ptr(),
                                             h.data_ptr(), ws.data_ptr(), ws.numel(), 16, 512, 48,
                                             None)
    assert st == 2  # DFL_ERR_BAD_SHAPE
    with pytest.raises(ValueError):
        pkg.gate_up_silu(x, w, s, s)
