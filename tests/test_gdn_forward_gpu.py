"""GPU parity of the GatedDeltaNet verify forward with tape recording
(``gated_delta_kernel_with_tape``, reference ``dflash_mlx/kernels.py:169-219``)
against the CPU oracle's restatement of ``_gated_delta_ops_with_tape``
(``kernels.py:125-167``).

Inputs follow BASELINE config 4 (k L2-normalised, v ~ N(0, 1),
beta = sigmoid(N), g = exp(-softplus(N)), S ~ N(0, 0.05)), with K-head
broadcast, vector decay, masks and T = 0.  Tolerances: state and tape
rel 1e-3 (atol 1e-4 / 1e-5); y (bf16) within two bf16 ulps of the oracle.
The dot-product sums run in a different order than numpy's, so agreement is
to tolerance; the forward -> replay identity between the two GPU kernels is
exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bf16 as obf16
from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu


def _inputs(seed, b, t, hk, hv, dk, dv, vec=False):
    rng = np.random.default_rng(seed)
    q = obf16.round_f32(rng.standard_normal((b, t, hk, dk)).astype(np.float32) / np.sqrt(dk))
    k = rng.standard_normal((b, t, hk, dk)).astype(np.float32)
    k = obf16.round_f32(k / np.linalg.norm(k, axis=-1, keepdims=True))
    v = obf16.round_f32(rng.standard_normal((b, t, hv, dv)).astype(np.float32))
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, t, hv))))).astype(np.float32)
    gshape = (b, t, hv, dk) if vec else (b, t, hv)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal(gshape)))).astype(np.float32)
    s0 = (rng.standard_normal((b, hv, dv, dk)) * 0.05).astype(np.float32)
    return q, k, v, g, beta, s0


def _dev(a, dev, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


def _run(pkg, dev, q, k, v, g, beta, s0, mask=None):
    bf = torch.bfloat16
    m = None if mask is None else torch.from_numpy(mask).to(dev)
    y, s1, tape = pkg.gated_delta_kernel_with_tape(
        _dev(q, dev, bf), _dev(k, dev, bf), _dev(v, dev, bf), _dev(g, dev, torch.float32),
        _dev(beta, dev, torch.float32), _dev(s0, dev, torch.float32), mask=m)
    return y.float().cpu().numpy(), s1.cpu().numpy(), tape.cpu().numpy()


def _check(got, ref):
    y, s1, tape = got
    ry, rs1, rtape = ref
    assert tape.dtype == np.float32 and s1.dtype == np.float32
    np.testing.assert_allclose(s1, rs1, rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(tape, rtape, rtol=1e-3, atol=1e-5)
    ry_bf = obf16.round_f32(ry)
    ulp = np.maximum(np.abs(ry_bf), 1e-3) * 2.0 ** -7
    assert np.all(np.abs(y - ry_bf) <= 2 * ulp + 1e-4)


@pytest.mark.parametrize("b,t,hk,hv,dk,dv,vec", [
    (2, 16, 16, 48, 128, 128, False),   # BASELINE config 4 heads, K-head broadcast 3:1
    (2, 16, 4, 4, 128, 64, True),       # vector decay
    (1, 7, 1, 2, 64, 32, False),        # ragged T, Dk 64
    (1, 5, 2, 2, 256, 32, True),        # Dk 256
    (3, 16, 1, 1, 32, 32, False),       # Dk 32
    (1, 9, 2, 2, 128, 96, True),        # Dk 128 with Dv % 64 != 0 (general kernel)
])
def test_forward_tape_matches_oracle(pkg, dev, b, t, hk, hv, dk, dv, vec):
    q, k, v, g, beta, s0 = _inputs(b * 100 + t + dk, b, t, hk, hv, dk, dv, vec)
    got = _run(pkg, dev, q, k, v, g, beta, s0)
    _check(got, ogdn.gated_delta_with_tape(q, k, v, g, beta, s0))


def test_forward_tape_with_mask(pkg, dev):
    b, t, hk, hv, dk, dv = 2, 12, 2, 4, 128, 64
    q, k, v, g, beta, s0 = _inputs(9, b, t, hk, hv, dk, dv)
    mask = np.ones((b, t), dtype=np.uint8)
    mask[0, 3] = mask[0, 9:] = 0
    mask[1, 0] = 0
    got = _run(pkg, dev, q, k, v, g, beta, s0, mask)
    _check(got, ogdn.gated_delta_with_tape(q, k, v, g, beta, s0, mask=mask.astype(bool)))
    assert np.all(got[2][0, 3] == 0) and np.all(got[2][0, 9:] == 0) and np.all(got[2][1, 0] == 0)


def test_forward_zero_steps_copies_state(pkg, dev):
    q, k, v, g, beta, s0 = _inputs(3, 2, 0, 2, 4, 64, 32)
    y, s1, tape = _run(pkg, dev, q, k, v, g, beta, s0)
    assert y.shape == (2, 0, 4, 32) and tape.shape == (2, 0, 4, 32)
    assert np.array_equal(s1, s0)


@pytest.mark.parametrize("vec", [False, True])
def test_replaying_the_tape_reproduces_the_forward_state_exactly(pkg, dev, vec):
    """Rollback contract (recurrent_rollback_cache.py:142-165): replaying the
    first a steps of the recorded tape onto the snapshot gives the state the
    forward reached after a steps, bit for bit (same operations, same order)."""
    b, t, hk, hv, dk, dv = 3, 16, 16, 48, 128, 128
    q, k, v, g, beta, s0 = _inputs(11 + vec, b, t, hk, hv, dk, dv, vec)
    bf = torch.bfloat16
    tq, tk, tv = (_dev(a, dev, bf) for a in (q, k, v))
    tg, tb, ts0 = (_dev(a, dev, torch.float32) for a in (g, beta, s0))
    _, _, tape = pkg.gated_delta_kernel_with_tape(tq, tk, tv, tg, tb, ts0)
    accepted = torch.tensor([0, 5, 16], dtype=torch.int32, device=dev)
    replayed = ts0.clone()
    pkg.tape_replay_(replayed, tape, tk, tg, accepted)
    for i, a in enumerate(accepted.tolist()):
        _, s_a, _ = pkg.gated_delta_kernel_with_tape(tq[i:i + 1, :a], tk[i:i + 1, :a], tv[i:i + 1, :a],
                                                     tg[i:i + 1, :a], tb[i:i + 1, :a], ts0[i:i + 1])
        assert torch.equal(replayed[i:i + 1], s_a), f"sequence {i}, a={a}"
