"""The pair-packed weight layout of the verify qmm.

``repack_pairs`` reorders each uint32's nibbles so that the kernel's
dequantiser yields natural K order; the qmm on repacked weights then reads x
by TMA without a permutation step.  Checks: the repack is bit-exact against
the oracle's restatement (and in place), and the qmm on repacked weights
matches the oracle on the original MLX weights with the same tolerance as
the MLX-layout path (|y - ref| <= 1e-2 + 2e-2 |ref|; reference harness
max_abs <= 8e-3 bf16 / 4e-3 fp16, max_rel <= 2e-2).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import bf16_to_np_bits, to_dev_bf16, to_dev_u32
from oracle import bf16 as obf16
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu


def _u32(t):
    import torch

    return t.detach().contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def _close(y_bits, ref_bits, what):
    y = obf16.to_f32(y_bits).astype(np.float64)
    r = obf16.to_f32(ref_bits).astype(np.float64)
    bad = np.abs(y - r) > 1e-2 + 2e-2 * np.abs(r)
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} outside tolerance"


def test_repack_matches_oracle_and_runs_in_place(pkg, dev):
    rng = np.random.default_rng(1)
    w_q = rng.integers(0, 2**32, size=(96, 128), dtype=np.uint64).astype(np.uint32)
    t = to_dev_u32(w_q, dev)
    out = pkg.repack_pairs(t)
    assert np.array_equal(_u32(out), oqmm.pair_pack(w_q))
    pkg.repack_pairs(t, out=t)
    assert np.array_equal(_u32(t), oqmm.pair_pack(w_q))


@pytest.mark.parametrize("M,K,N", [
    (16, 4096, 4096),     # BASELINE config 0 shape
    (16, 5120, 17408),    # gate_proj
    (16, 17408, 5120),    # down_proj
    (4, 5120, 17408),
    (32, 4096, 1024),     # MT = 32
    (17, 1600, 384),      # ragged M, K % 512 != 0
    (16, 640, 200),       # ragged N, K tail
    (1, 64, 8),
    (3, 8192, 136),
    (16, 512, 128 * 740),  # many one-unit tiles per CTA
    (16, 2560, 128 * 160),
    (32, 512, 128 * 600),
])
def test_pairs_layout_matches_oracle(pkg, dev, M, K, N):
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    w_q, s, b = oqmm.synth_weights(rng, N, K)
    x = oqmm.synth_x(rng, M, K)
    wp = pkg.repack_pairs(to_dev_u32(w_q, dev))
    y = pkg.qmm_w4g64(to_dev_bf16(x, dev), wp, to_dev_bf16(s, dev), to_dev_bf16(b, dev),
                      layout="pairs")
    ref = oqmm.qmm(x, w_q, s, b, accum=np.float32)
    _close(bf16_to_np_bits(y), ref, f"{M}x{K}x{N}")


def test_pairs_dequant_is_exact(pkg, dev):
    rng = np.random.default_rng(3)
    k, n = 1024, 256
    w_q, s, b = oqmm.synth_weights(rng, n, k)
    cols = rng.choice(k, size=16, replace=False)
    xf = np.zeros((16, k), dtype=np.float32)
    xf[np.arange(16), cols] = 1.0
    wp = pkg.repack_pairs(to_dev_u32(w_q, dev))
    y = pkg.qmm_w4g64(to_dev_bf16(obf16.from_f32(xf), dev), wp, to_dev_bf16(s, dev),
                      to_dev_bf16(b, dev), layout="pairs")
    w = oqmm.dequantize(w_q, s, b)
    assert np.array_equal(obf16.to_f32(bf16_to_np_bits(y)), w[:, cols].T)


def test_pairs_reference_harness_bf16_and_f16(pkg, dev):
    import torch

    for dtype, tol in (("bf16", 8e-3), ("f16", 4e-3)):
        rng = np.random.default_rng(17)
        M, K, N = 16, 5120, 6144
        scale = 1.0 / np.sqrt(K)
        if dtype == "bf16":
            x = obf16.from_f32((rng.standard_normal((M, K)) * scale).astype(np.float32))
            w = obf16.round_f32((rng.standard_normal((N, K)) * scale).astype(np.float32))
            tdt = torch.bfloat16
        else:
            x = (rng.standard_normal((M, K)) * scale).astype(np.float16).view(np.uint16)
            w = (rng.standard_normal((N, K)) * scale).astype(np.float16).astype(np.float32)
            tdt = torch.float16
        w_q, s, b = oqmm.affine_quantize(w, dtype=dtype)

        def dev16(a):
            return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(tdt)

        wp = pkg.repack_pairs(to_dev_u32(w_q, dev))
        y = pkg.qmm_w4g64(dev16(x), wp, dev16(s), dev16(b), layout="pairs")
        ybits = y.view(torch.int16).cpu().numpy().view(np.uint16)
        ref = oqmm.qmm(x, w_q, s, b, accum=np.float32, dtype=dtype)
        max_abs, max_rel = oqmm.max_abs_rel(ybits, ref, dtype=dtype)
        assert max_abs <= tol and max_rel <= 2e-2, (dtype, max_abs, max_rel)


def test_pairs_deterministic(pkg, dev):
    rng = np.random.default_rng(11)
    w_q, s, b = oqmm.synth_weights(rng, 1024, 6144)
    x = to_dev_bf16(oqmm.synth_x(rng, 16, 6144), dev)
    wp = pkg.repack_pairs(to_dev_u32(w_q, dev))
    sd, bd = to_dev_bf16(s, dev), to_dev_bf16(b, dev)
    y1 = pkg.qmm_w4g64(x, wp, sd, bd, layout="pairs")
    y2 = pkg.qmm_w4g64(x, wp, sd, bd, layout="pairs")
    assert bf16_to_np_bits(y1).tobytes() == bf16_to_np_bits(y2).tobytes()
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0
