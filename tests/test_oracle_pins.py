"""Pins the CPU oracle to the reference's own golden cases (CPU only).

* acceptance: ``tests/test_engine_acceptance.py:11-24`` (exact table);
* tape replay: ``tests/test_gated_delta_tree_kernel.py:162-178`` -- replaying
  the tree tape along the accepted slots [0, 1, 3] equals the tree state at
  slot 3 (atol 1e-4), on the arange inputs of ``:22-54``; and the tape-kernel
  dtype checks of ``:98-160`` (tape stays fp32 with bf16 inputs);
* qmm nibble layout: hand-computed known answers for
  ``dflash_mlx/verify_qmm.py:243-250`` (nibble ki of word p is column 8p+ki).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import bf16 as obf16
from oracle import gdn as ogdn
from oracle import lmhead as olm
from oracle import qmm as oqmm


@pytest.mark.parametrize("drafted,posterior,expected", [
    ([], [], 0),
    ([1, 2, 3, 4], [1, 2, 3, 4], 4),
    ([5, 5, 5], [1, 5, 5], 0),
    ([1, 2, 9, 4, 5], [1, 2, 3, 4, 5], 2),
    ([7, 7, 7, 0], [7, 7, 7, 1], 3),
])
def test_acceptance_golden_table(drafted, posterior, expected):
    assert olm.match_acceptance_length(np.array(drafted, np.uint32),
                                       np.array(posterior, np.uint32)) == expected


def _tree_inputs(vectorized_g: bool):
    # tests/test_gated_delta_tree_kernel.py:22-54
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
def test_replay_along_accepted_path_equals_tree_state(vec):
    q, k, v, g, beta, state, parent = _tree_inputs(vec)
    _, tape = ogdn.gated_delta_tree_tape(q, k, v, g, beta, state, parent)
    _, states = ogdn.gated_delta_tree(q, k, v, g, beta, state, parent)
    slots = [0, 1, 3]
    replayed = ogdn.tape_replay(tape[:, slots], k[:, slots], g[:, slots], state)
    assert np.max(np.abs(replayed - states[:, 3])) <= 1e-4
    assert tape.dtype == np.float32


def test_linear_tape_replay_reproduces_forward_state():
    # replaying all T steps of a linear (chain) tape rebuilds the final state,
    # and replaying a prefix rebuilds the intermediate state (rollback contract,
    # recurrent_rollback_cache.py:142-165)
    rng = np.random.default_rng(0)
    b, t, hk, hv, dk, dv = 2, 6, 2, 4, 32, 8
    q = rng.standard_normal((b, t, hk, dk)).astype(np.float32)
    k = rng.standard_normal((b, t, hk, dk)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((b, t, hv, dv)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, t, hv))))).astype(np.float32)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal((b, t, hv))))).astype(np.float32)
    s0 = (rng.standard_normal((b, hv, dv, dk)) * 0.05).astype(np.float32)
    _, s_final, tape = ogdn.gated_delta_with_tape(q, k, v, g, beta, s0)
    full = ogdn.tape_replay(tape, k, g, s0)
    assert np.allclose(full, s_final, atol=1e-5, rtol=1e-4)
    for a in range(t + 1):
        _, s_a, _ = ogdn.gated_delta_with_tape(q[:, :a], k[:, :a], v[:, :a], g[:, :a],
                                               beta[:, :a], s0)
        rep = ogdn.tape_replay_accepted(tape, k, g, s0, np.full(b, a))
        assert np.allclose(rep, s_a, atol=1e-5, rtol=1e-4)


def test_tape_stays_fp32_with_bf16_inputs():
    q, k, v, g, beta, state, _ = _tree_inputs(False)
    rb = obf16.round_f32
    _, s1, tape = ogdn.gated_delta_with_tape(rb(q), rb(k), rb(v), rb(g), rb(beta), state)
    assert tape.dtype == np.float32 and s1.dtype == np.float32


def test_nibble_layout_known_answer():
    # word 0 = 0x76543210 holds columns 0..7 with values 0..7, low nibble first
    w_q = np.array([[0x76543210, 0xFEDCBA98]], dtype=np.uint32)
    assert oqmm.unpack_nibbles(w_q).tolist() == [list(range(16))]
    assert np.array_equal(oqmm.pack_nibbles(oqmm.unpack_nibbles(w_q)), w_q)


def test_dequant_and_qmm_known_answer():
    # K = 64 (one group), N = 2 rows; scale 0.5 / bias -2 on row 0, scale 1 / bias 0 on row 1
    nib = np.zeros((2, 64), dtype=np.uint8)
    nib[0, :16] = np.arange(16)
    nib[1, :] = 3
    w_q = oqmm.pack_nibbles(nib)
    s = obf16.from_f32(np.array([[0.5], [1.0]], np.float32))
    b = obf16.from_f32(np.array([[-2.0], [0.0]], np.float32))
    w = oqmm.dequantize(w_q, s, b)
    assert w[0, :16].tolist() == [0.5 * i - 2.0 for i in range(16)]
    assert np.all(w[0, 16:] == -2.0) and np.all(w[1] == 3.0)
    x = obf16.from_f32(np.ones((1, 64), np.float32))
    y = obf16.to_f32(oqmm.qmm(x, w_q, s, b))
    # row 0: sum(0.5 i - 2, i < 16) + 48 * (-2) = 60 - 32 - 96 = -68; row 1: 64 * 3 = 192
    assert y.tolist() == [[-68.0, 192.0]]


def test_vocab_split_reduce_matches_global_argmax():
    rng = np.random.default_rng(5)
    logits = obf16.round_f32(rng.standard_normal((32, 1000)).astype(np.float32))
    logits[3, 10] = logits[3, 700] = 50.0   # tie across shards -> lower index
    bounds = [0, 250, 500, 750, 1000]
    vals, idxs = [], []
    for g in range(4):
        v, i = olm.shard_partials(logits[:, bounds[g]:bounds[g + 1]], bounds[g])
        vals.append(v)
        idxs.append(i)
    assert np.array_equal(olm.reduce_partials(np.stack(vals), np.stack(idxs)),
                          np.argmax(logits, axis=-1))


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.0e-41, np.inf], dtype=np.float32)
    r = obf16.round_f32(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.015625 and np.isinf(r[4])
