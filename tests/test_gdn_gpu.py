"""GPU parity of the GatedDeltaNet tape replay against the CPU oracle.

Cases follow the reference's GDN tests (``tests/test_gated_delta_tree_kernel.py``):
the arange inputs of ``:22-54`` and the replay-equals-tree-state identity of
``:162-178`` (atol 1e-4), plus BASELINE config 4 shapes (Hv = 48, Dk = Dv =
128, T = 16, bf16 k, per-sequence accepted step counts 0..16) with K-head
broadcast (Hk = 16) and vector decay.  The kernel applies the mx-op
reference's two separately rounded fp32 updates per step, so against the
oracle it is bit-exact; the stated tolerance (rel 1e-3) is checked as well.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bf16 as obf16
from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


def _tree_inputs(vectorized_g):
    b, t, hk, hv, dk, dv = 1, 4, 1, 2, 32, 4
    q = np.arange(b * t * hk * dk, dtype=np.float32).reshape(b, t, hk, dk) / 100.0
    k = (np.arange(b * t * hk * dk, dtype=np.float32) + 3).reshape(b, t, hk, dk) / 110.0
    v = (np.arange(b * t * hv * dv, dtype=np.float32) + 5).reshape(b, t, hv, dv) / 20.0
    beta = np.full((b, t, hv), 0.25, dtype=np.float32)
    state = np.zeros((b, hv, dv, dk), dtype=np.float32)
    parent = np.array([-1, 0, 1, 1], dtype=np.int32)
    g = np.full((b, t, hv, dk) if vectorized_g else (b, t, hv), 0.91, dtype=np.float32)
    return q, k, v, g, beta, state, parent


@pytest.mark.parametrize("vec", [False, True])
def test_replay_accepted_tree_path_equals_tree_state(pkg, dev, vec):
    q, k, v, g, beta, state, parent = _tree_inputs(vec)
    _, tape = ogdn.gated_delta_tree_tape(q, k, v, g, beta, state, parent)
    _, states = ogdn.gated_delta_tree(q, k, v, g, beta, state, parent)
    slots = [0, 1, 3]
    out = pkg.tape_replay_kernel(_t(tape[:, slots], dev), _t(k[:, slots], dev),
                                 _t(g[:, slots], dev), _t(state, dev)).cpu().numpy()
    assert np.max(np.abs(out - states[:, 3])) <= 1e-4


def _config4(seed, b, hv, hk, d, t, vec):
    rng = np.random.default_rng(seed)
    s0 = (rng.standard_normal((b, hv, d, d)) * 0.05).astype(np.float32)
    kk = rng.standard_normal((b, t, hk, d)).astype(np.float32)
    kk = obf16.round_f32(kk / np.linalg.norm(kk, axis=-1, keepdims=True))
    tape = rng.standard_normal((b, t, hv, d)).astype(np.float32) * 0.3
    shape = (b, t, hv, d) if vec else (b, t, hv)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal(shape)))).astype(np.float32)
    steps = rng.integers(0, t + 1, size=b).astype(np.int32)
    return s0, kk, tape, g, steps


@pytest.mark.parametrize("hk,vec", [(48, False), (16, False), (48, True)])
def test_config4_shapes_bit_exact_inplace(pkg, dev, hk, vec):
    b, hv, d, t = 6, 48, 128, 16
    s0, kk, tape, g, steps = _config4(7 + hk, b, hv, hk, d, t, vec)
    steps[0] = 0
    steps[1] = t
    ref = ogdn.tape_replay_accepted(tape, kk, g, s0, steps)
    st = _t(s0, dev)
    pkg.kernels.tape_replay_(st, _t(tape, dev), _t(kk, dev, torch.bfloat16), _t(g, dev),
                             torch.from_numpy(steps))
    out = st.cpu().numpy()
    assert np.array_equal(out, ref)
    rel = np.abs(out - ref) / (np.abs(ref) + 1e-6)
    assert rel.max() <= 1e-3
    assert np.array_equal(out[0], s0[0])  # nothing replayed: untouched


def test_functional_form_with_mask_matches_oracle(pkg, dev):
    b, hv, hk, d, t = 3, 8, 4, 64, 12
    s0, kk, tape, g, _ = _config4(3, b, hv, hk, d, t, False)
    rng = np.random.default_rng(9)
    mask = rng.random((b, t)) < 0.6
    ref = ogdn.tape_replay(tape, kk, g, s0, mask)
    s_in = _t(s0, dev)
    out = pkg.tape_replay_kernel(_t(tape, dev), _t(kk, dev), _t(g, dev), s_in,
                                 torch.from_numpy(mask)).cpu().numpy()
    assert np.array_equal(out, ref)
    assert np.array_equal(s_in.cpu().numpy(), s0)  # functional: input untouched


def test_rollback_cache_replays_accepted_plus_one(pkg, dev):
    # arm -> (verify writes the post-block state) -> rollback(n) == replay of n + 1 steps
    b, hv, hk, d, t = 2, 4, 4, 32, 8
    rng = np.random.default_rng(1)
    q = rng.standard_normal((b, t, hk, d)).astype(np.float32)
    kk = rng.standard_normal((b, t, hk, d)).astype(np.float32)
    kk /= np.linalg.norm(kk, axis=-1, keepdims=True)
    v = rng.standard_normal((b, t, hv, d)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, t, hv))))).astype(np.float32)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal((b, t, hv))))).astype(np.float32)
    s0 = (rng.standard_normal((b, hv, d, d)) * 0.05).astype(np.float32)
    _, s_final, tape = ogdn.gated_delta_with_tape(q, kk, v, g, beta, s0)
    qkv = rng.standard_normal((b, t, 24)).astype(np.float32)
    cache = pkg.RecurrentRollbackCache(2, conv_kernel_size=4)
    cache[0] = _t(np.zeros((b, 3, 24), np.float32), dev)
    cache[1] = _t(s0, dev)
    cache.arm_rollback(prefix_len=10)
    cache[1] = _t(s_final, dev)
    cache.record_tape(tape=_t(tape, dev), k=_t(kk, dev), g=_t(g, dev), qkv=_t(qkv, dev))
    cache.rollback(2)
    _, s3, _ = ogdn.gated_delta_with_tape(q[:, :3], kk[:, :3], v[:, :3], g[:, :3], beta[:, :3], s0)
    assert np.allclose(cache[1].cpu().numpy(), s3, atol=1e-5, rtol=1e-4)
    conv = np.concatenate([np.zeros((b, 3, 24), np.float32), qkv], axis=1)[:, 3:6]
    assert np.array_equal(cache[0].cpu().numpy(), conv)
    assert cache._snapshot is None and cache._tape is None
