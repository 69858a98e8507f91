"""DDTree verify kernels on the GPU against the CPU oracle.

Cases follow the reference's ``tests/test_gated_delta_tree_kernel.py``: the
arange inputs of ``:22-54`` (B=1, T=4, Hk=1, Hv=2, Dk=32, Dv=4, parents
[-1, 0, 1, 1]) with scalar and vector decay and its tolerances (atol 1e-4,
1e-5 for fp32 states from bf16 inputs); the tree tape replayed along the
accepted slots [0, 1, 3] equals the tree state of node 3 (``:162-178``); the
tree conv1d inputs of ``:181-214``.  On top: random trees at Qwen3.6-27B GDN
head sizes (Hv=48 shared by Hk=16 k heads is scaled to Hv=8, Hk=4 here,
Dk=Dv=128), bf16 inputs, y within bf16 rounding (1e-2 + 2e-2|ref|) and
states rel 1e-3; and bad parent ids / path slots recorded as a device error.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu


def _ref_inputs(vectorized_g, dtype="f32"):
    import torch

    b, t, hk, hv, dk, dv = 1, 4, 1, 2, 32, 4
    q = np.arange(b * t * hk * dk, dtype=np.float32).reshape(b, t, hk, dk) / 100.0
    k = (np.arange(b * t * hk * dk, dtype=np.float32) + 3).reshape(b, t, hk, dk) / 110.0
    v = (np.arange(b * t * hv * dv, dtype=np.float32) + 5).reshape(b, t, hv, dv) / 20.0
    beta = np.full((b, t, hv), 0.25, np.float32)
    state = np.zeros((b, hv, dv, dk), np.float32)
    parent = np.array([-1, 0, 1, 1], np.int32)
    g = np.full((b, t, hv, dk) if vectorized_g else (b, t, hv), 0.91, np.float32)
    if dtype == "bf16":
        q, k, v, g, beta = (torch.from_numpy(a).to(torch.bfloat16).float().numpy() for a in (q, k, v, g, beta))
    return q, k, v, g, beta, state, parent


def _dev(a, dev, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


@pytest.mark.parametrize("vec", [False, True])
def test_tree_matches_reference_ops_f32(pkg, dev, vec):
    q, k, v, g, beta, state, parent = _ref_inputs(vec)
    y, states = pkg.gated_delta_tree_kernel(*(_dev(a, dev) for a in (q, k, v, g, beta, state, parent)))
    ey, es = ogdn.gated_delta_tree(q, k, v, g, beta, state, parent)
    assert np.max(np.abs(y.cpu().numpy() - ey)) <= 1e-4
    assert np.max(np.abs(states.cpu().numpy() - es)) <= 1e-4


def test_tree_keeps_state_dtype_with_bf16_inputs(pkg, dev):
    import torch

    q, k, v, g, beta, state, parent = _ref_inputs(False, "bf16")
    ins = [_dev(q, dev, torch.bfloat16), _dev(k, dev, torch.bfloat16), _dev(v, dev, torch.bfloat16),
           _dev(g, dev, torch.bfloat16), _dev(beta, dev, torch.bfloat16), _dev(state, dev), _dev(parent, dev)]
    _, states = pkg.gated_delta_tree_kernel(*ins)
    _, es = ogdn.gated_delta_tree(q, k, v, g, beta, state, parent)
    assert states.dtype == torch.float32
    assert np.max(np.abs(states.cpu().numpy() - es)) <= 1e-5


def test_tree_tape_bf16_and_replay_of_accepted_path(pkg, dev):
    import torch

    q, k, v, g, beta, state, parent = _ref_inputs(False, "bf16")
    qd, kd, vd = (_dev(a, dev, torch.bfloat16) for a in (q, k, v))
    gd, bd, sd, pd = _dev(g, dev), _dev(beta, dev), _dev(state, dev), _dev(parent, dev)
    y, tape = pkg.gated_delta_tree_tape_kernel(qd, kd, vd, gd, bd, sd, pd)
    ey, etape = ogdn.gated_delta_tree_tape(q, k, v, g, beta, state, parent)
    assert tape.dtype == torch.float32
    yv = y.float().cpu().numpy()
    assert not (np.abs(yv - ey) > 1e-2 + 2e-2 * np.abs(ey)).any()  # bf16 output rounding
    assert np.max(np.abs(tape.cpu().numpy() - etape)) <= 1e-5
    _, states = pkg.gated_delta_tree_kernel(qd, kd, vd, gd, bd, sd, pd)
    acc = torch.tensor([0, 1, 3], device=dev)
    replayed = pkg.tape_replay_kernel(tape[:, acc].contiguous(), kd[:, acc].contiguous(),
                                      gd[:, acc].contiguous(), sd)
    assert torch.equal(replayed, states[:, 3])


def _random_tree(rng, t):
    parent = np.empty(t, np.int32)
    parent[0] = -1
    for i in range(1, t):
        parent[i] = int(rng.integers(-1, i))
    return parent


@pytest.mark.parametrize("vec", [False, True])
def test_random_trees_at_model_head_sizes(pkg, dev, vec):
    import torch

    rng = np.random.default_rng(31 + vec)
    b, t, hk, hv, dk, dv = 2, 16, 4, 8, 128, 128

    def unit(shape):
        a = rng.standard_normal(shape).astype(np.float32)
        return a / np.linalg.norm(a, axis=-1, keepdims=True)

    q = torch.from_numpy(unit((b, t, hk, dk))).to(torch.bfloat16)
    k = torch.from_numpy(unit((b, t, hk, dk))).to(torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((b, t, hv, dv)).astype(np.float32)).to(torch.bfloat16)
    gshape = (b, t, hv, dk) if vec else (b, t, hv)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal(gshape)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((b, t, hv))))).astype(np.float32)
    state = (rng.standard_normal((b, hv, dv, dk)) * 0.05).astype(np.float32)
    parent = _random_tree(rng, t)
    y, states = pkg.gated_delta_tree_kernel(q.to(dev), k.to(dev), v.to(dev), _dev(g, dev), _dev(beta, dev),
                                            _dev(state, dev), _dev(parent, dev))
    ey, es = ogdn.gated_delta_tree(q.float().numpy(), k.float().numpy(), v.float().numpy(), g, beta, state,
                                   parent)
    yv = y.float().cpu().numpy()
    assert not (np.abs(yv - ey) > 1e-2 + 2e-2 * np.abs(ey)).any()
    sv = states.cpu().numpy()
    assert np.max(np.abs(sv - es)) <= 1e-3 * max(1.0, float(np.max(np.abs(es))))


def test_tree_conv1d_matches_reference_ops(pkg, dev):
    import torch

    b, t, c, kk = 1, 4, 6, 4
    qkv = np.arange(b * t * c, dtype=np.float32).reshape(b, t, c) / 100.0
    prefix = (np.arange(b * (kk - 1) * c, dtype=np.float32) + 2).reshape(b, kk - 1, c) / 90.0
    weight = (np.arange(c * kk, dtype=np.float32) + 1).reshape(c, kk, 1) / 80.0
    path = np.array([[0, 1, 2, 3], [1, 2, 3, 4], [1, 2, 3, 5], [2, 3, 4, 6]], np.int32)
    out = pkg.tree_depthwise_conv1d(_dev(qkv, dev), _dev(prefix, dev), _dev(weight, dev), None, _dev(path, dev))
    exp = ogdn.tree_depthwise_conv1d(qkv, prefix, weight, None, path)
    assert np.max(np.abs(out.cpu().numpy() - exp)) <= 1e-4
    # bf16 with bias, wider channels
    rng = np.random.default_rng(4)
    b, t, c = 2, 8, 512
    qkv = rng.standard_normal((b, t, c)).astype(np.float32)
    prefix = rng.standard_normal((b, kk - 1, c)).astype(np.float32)
    w = (rng.standard_normal((c, kk, 1)) * 0.3).astype(np.float32)
    bias = (rng.standard_normal(c) * 0.1).astype(np.float32)
    path = np.stack([np.arange(i, i + kk) for i in range(t)]).astype(np.int32)
    qb = torch.from_numpy(qkv).to(torch.bfloat16)
    pb = torch.from_numpy(prefix).to(torch.bfloat16)
    out = pkg.tree_depthwise_conv1d(qb.to(dev), pb.to(dev), _dev(w, dev), _dev(bias, dev), _dev(path, dev))
    exp = ogdn.tree_depthwise_conv1d(qb.float().numpy(), pb.float().numpy(), w, bias, path)
    ov = out.float().cpu().numpy()
    assert not (np.abs(ov - exp) > 1e-2 + 2e-2 * np.abs(exp)).any()


def test_bad_parent_and_slot_are_reported(pkg, dev):
    from dflash_mlx_b200 import _lib

    assert _lib.device_error() == 0
    q, k, v, g, beta, state, _ = _ref_inputs(False)
    bad = np.array([-1, 0, 3, 1], np.int32)  # node 2 names a later node
    pkg.gated_delta_tree_kernel(*(_dev(a, dev) for a in (q, k, v, g, beta, state, bad)))
    assert _lib.device_error() == 3
    qkv = np.zeros((1, 2, 4), np.float32)
    prefix = np.zeros((1, 1, 4), np.float32)
    w = np.ones((4, 2, 1), np.float32)
    path = np.array([[0, 1], [1, 7]], np.int32)  # slot 7 is outside [0, 3)
    pkg.tree_depthwise_conv1d(_dev(qkv, dev), _dev(prefix, dev), _dev(w, dev), None, _dev(path, dev))
    assert _lib.device_error() == 3
    assert _lib.device_error() == 0
