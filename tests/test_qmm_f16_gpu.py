"""GPU parity of the fp16-activation verify qmm against the CPU oracle.

The reference builds an fp16 kernel beside the bf16 one for every verify
linear (``dflash_mlx/verify_linear.py:163-164``) and its parity harness runs
the real MLP shapes in both dtypes (``tests/test_verify_qmm_parity.py:74-94``)
with max_abs <= 4e-3 for fp16 and max_rel <= 2e-2.  Inputs follow that
harness: x, w ~ N(0,1)/sqrt(K) in fp16, w quantised to 4 bits with fp16
scales and biases.  The oracle rounds each dequantised weight to fp16 and
accumulates in fp32, as the kernel does.
"""

from __future__ import annotations

import zlib
import numpy as np
import pytest

from conftest import to_dev_u32
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu


def _to_dev_f16(a, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.float16)


def _bits(t):
    import torch

    assert t.dtype == torch.float16
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _f16_case(name, M, K, N):
    rng = np.random.default_rng(zlib.crc32(f"{name}-{M}-{K}-{N}-f16".encode()) & 0xFFFF)
    scale = 1.0 / np.sqrt(max(K, 1))
    x = (rng.standard_normal((M, K)) * scale).astype(np.float16).view(np.uint16)
    w = (rng.standard_normal((N, K)) * scale).astype(np.float16).astype(np.float32)
    w_q, s, b = oqmm.affine_quantize(w, dtype="f16")
    return x, w_q, s, b


def _run(pkg, dev, x, w_q, s, b):
    y = pkg.verify_matmul(_to_dev_f16(x, dev), to_dev_u32(w_q, dev), _to_dev_f16(s, dev),
                          _to_dev_f16(b, dev))
    return _bits(y)


@pytest.mark.parametrize("name,M,K,N", [
    ("gate_proj", 16, 5120, 17408),
    ("down_proj", 16, 17408, 5120),
    ("gate_proj_m4", 4, 5120, 17408),
    ("down_proj_m4", 4, 17408, 5120),
    ("mt32", 32, 4096, 1024),
    ("plain_sb", 17, 1600, 384),      # K % 512 != 0: scales/biases by plain loads
    ("tiny", 1, 64, 8),
])
def test_f16_reference_harness(pkg, dev, name, M, K, N):
    x, w_q, s, b = _f16_case(name, M, K, N)
    y = _run(pkg, dev, x, w_q, s, b)
    ref = oqmm.qmm(x, w_q, s, b, accum=np.float32, dtype="f16")
    assert y.shape == (M, N)
    max_abs, max_rel = oqmm.max_abs_rel(y, ref, dtype="f16")
    assert max_abs <= 4e-3 and max_rel <= 2e-2, (name, max_abs, max_rel)


def test_f16_dequant_is_exact(pkg, dev):
    # one-hot fp16 activations pick single dequantised weights: y[m, n] = w[n, k_m]
    rng = np.random.default_rng(5)
    k, n = 1024, 256
    w_q, s, b = oqmm.synth_weights(rng, n, k, dtype="f16")
    cols = rng.choice(k, size=16, replace=False)
    xf = np.zeros((16, k), dtype=np.float16)
    xf[np.arange(16), cols] = 1.0
    y = _run(pkg, dev, xf.view(np.uint16), w_q, s, b)
    w = oqmm.dequantize(w_q, s, b, dtype="f16")
    assert np.array_equal(y.view(np.float16).astype(np.float32), w[:, cols].T)


def test_f16_and_bf16_entry_points_are_distinct(pkg, dev):
    """Same weights bits through both entry points give each dtype's own result."""
    import torch

    rng = np.random.default_rng(9)
    w_q, s, b = oqmm.synth_weights(rng, 512, 1024, dtype="f16")
    x = oqmm.synth_x(rng, 16, 1024, dtype="f16")
    y16 = _run(pkg, dev, x, w_q, s, b)
    ref = oqmm.qmm(x, w_q, s, b, accum=np.float32, dtype="f16")
    max_abs, _ = oqmm.max_abs_rel(y16, ref, dtype="f16")
    assert max_abs <= 4e-3
    with pytest.raises(NotImplementedError):
        pkg.verify_matmul(_to_dev_f16(x, dev), to_dev_u32(w_q, dev),
                          _to_dev_f16(s, dev).view(torch.bfloat16), _to_dev_f16(b, dev))
