"""GPU parity of the MoE verify layer run as one projection plan (grouped
plan phases over a sorted route table) against the CPU oracle.

Same restatement and tolerance as ``test_moe_gpu.py`` (mlx-lm's SwitchGLU ->
mx.gather_qmm, not vendored in the reference; |y - ref| <= 1e-2 + 2e-2 |ref|
+ 2^-7 max_row |ref|, bf16 out, fp32 accumulate).  Covered: the sorted route table and row gather
against a numpy sort of the same top-k ids, a small layer with ragged expert
loads, a layer where one expert takes every token, BASELINE config 2 (256
experts, top-8, hidden 2048, intermediate 512, shared expert, 16 tokens),
repeated calls on new inputs through the same plan (and a CUDA graph of
it), agreement with the per-launch MoE path, the fused route + sort launch
against the two separate ones (bit for bit), and out-of-range expert ids
(device error word set, empty table, nothing read out of bounds).  The
layer's down phase waits per expert problem for that problem's gate/up
tiles (per-problem counters), so every layer test also covers those waits.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_to_np_bits
from test_moe_gpu import _assert_close, _layer, _oracle

pytestmark = pytest.mark.gpu


def _numpy_sort(ids: np.ndarray):
    """Pairs ordered by expert id, then pair index -> (sorted pair rows,
    problem starts, problem experts)."""
    flat = ids.reshape(-1)
    order = sorted(range(flat.size), key=lambda p: (int(flat[p]), p))
    experts = sorted(set(int(e) for e in flat))
    starts = [int(np.searchsorted(np.sort(flat), e)) for e in experts]
    return np.array(order), starts, experts


def test_sort_pairs_table_and_rows(pkg, dev):
    gen = torch.Generator(device=dev).manual_seed(11)
    t, e, k, h = 16, 256, 8, 2048
    logits = torch.randn((t, e), generator=gen, device=dev)
    x = torch.randn((t, h), generator=gen, device=dev).to(torch.bfloat16)
    _, _, ids = pkg.moe.route(logits, k)
    x_copy = torch.zeros_like(x)
    route, xs = pkg.moe.sort_pairs(ids, x, e, x_copy=x_copy)
    order, starts, experts = _numpy_sort(ids.cpu().numpy())
    r = route.cpu().numpy()
    p = int(r[0])
    assert p == len(experts)
    assert [int(v) for v in r[1:1 + 2 * p:2]] == starts
    assert int(r[1 + 2 * p]) == t * k
    assert [int(v) for v in r[2:2 + 2 * p:2]] == experts
    assert np.array_equal(r[514:514 + t * k], order)
    assert torch.equal(xs, x[torch.as_tensor(order // k, device=dev)])
    assert torch.equal(x_copy, x)
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


@pytest.mark.parametrize("t,e,k", [(16, 256, 8), (5, 64, 4), (16, 4096, 16)])
def test_route_sorted_equals_route_then_sort(pkg, dev, t, e, k):
    """The fused launch gives route()'s ids and weights bit for bit and
    sort_pairs()'s table, rows and x copy."""
    gen = torch.Generator(device=dev).manual_seed(t * 1000 + e + k)
    logits = torch.randn((t, e), generator=gen, device=dev)
    logits[0, :8] = 1.5   # ties go to the lower expert id
    h = 256
    x = torch.randn((t, h), generator=gen, device=dev).to(torch.bfloat16)
    _, w_ref, ids_ref = pkg.moe.route(logits, k)
    route_ref, xs_ref = pkg.moe.sort_pairs(ids_ref, x, e)
    route = torch.full_like(route_ref, -7)
    xs = torch.zeros_like(xs_ref)
    x_copy = torch.zeros_like(x)
    w, ids = pkg.moe.route_sorted(logits, x, k, route_out=route, x_sorted=xs, x_copy=x_copy)
    assert torch.equal(ids, ids_ref)
    assert torch.equal(w.view(torch.int32), w_ref.view(torch.int32))
    p = int(route_ref[0].item())
    n = t * k
    assert torch.equal(route[:2 + 2 * p], route_ref[:2 + 2 * p])
    assert torch.equal(route[514:514 + n], route_ref[514:514 + n])
    assert torch.equal(xs, xs_ref) and torch.equal(x_copy, x)
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_route_sorted_appends_the_shared_expert(pkg, dev):
    """shared_expert=True: one more problem, expert E, over the T tokens
    themselves (sorted rows T*k + t = x[t], mapped to pair rows T*k + t)."""
    gen = torch.Generator(device=dev).manual_seed(12)
    t, e, k, h = 16, 256, 8, 512
    logits = torch.randn((t, e), generator=gen, device=dev)
    x = torch.randn((t, h), generator=gen, device=dev).to(torch.bfloat16)
    _, w_ref, ids_ref = pkg.moe.route(logits, k)
    route_ref, xs_ref = pkg.moe.sort_pairs(ids_ref, x, e)
    route = torch.full_like(route_ref, -7)
    xs = torch.zeros((t * k + t, h), dtype=torch.bfloat16, device=dev)
    w, ids = pkg.moe.route_sorted(logits, x, k, route_out=route, x_sorted=xs, shared_expert=True)
    assert torch.equal(ids, ids_ref) and torch.equal(w.view(torch.int32), w_ref.view(torch.int32))
    p = int(route_ref[0].item())
    n = t * k
    r = route.cpu().numpy()
    assert int(r[0]) == p + 1
    assert np.array_equal(r[1:2 + 2 * p], route_ref[1:2 + 2 * p].cpu().numpy())
    assert (int(r[1 + 2 * p]), int(r[2 + 2 * p]), int(r[3 + 2 * p])) == (n, e, n + t)
    assert np.array_equal(r[514:514 + n], route_ref[514:514 + n].cpu().numpy())
    assert np.array_equal(r[514 + n:514 + n + t], np.arange(n, n + t))
    assert torch.equal(xs[:n], xs_ref) and torch.equal(xs[n:], x)
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_moe_plan_layer_with_a_shared_expert_of_another_size(pkg, dev):
    """A shared expert whose intermediate size differs from the routed
    experts' runs as two dense phases of the same plan: same layer output as
    the oracle."""
    x, logits, experts, _ = _layer(pkg, dev, 8, 16, 32, 512, 256, 4, shared=False)
    gen = torch.Generator(device=dev).manual_seed(9)
    from test_moe_gpu import _qweight
    W = pkg.moe.QuantWeight
    sh = {name: W(*_qweight(gen, dev, (), n, kk))
          for name, n, kk in (("gate", 128, 512), ("up", 128, 512), ("down", 512, 128))}
    layer = pkg.moe.MoEPlanLayer(experts, sh, tokens=16, top_k=4)
    assert not layer.shared_stacked
    y = layer(x, logits)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, 4))
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_sort_pairs_rejects_out_of_range_ids(pkg, dev):
    """An expert id >= E sets the device error word and leaves an empty
    table (P = 0): no grouped phase then reads any weight."""
    from dflash_mlx_b200 import _lib

    assert _lib.device_error() == 0
    ids = torch.zeros((4, 2), dtype=torch.int32, device=dev)
    ids[2, 1] = 8
    x = torch.ones((4, 64), dtype=torch.bfloat16, device=dev)
    route, _ = pkg.moe.sort_pairs(ids, x, 8)
    assert int(route[0].item()) == 0
    assert _lib.device_error() == 3


@pytest.mark.parametrize("case", ["small", "one_expert", "config2"])
def test_moe_plan_layer_matches_oracle(pkg, dev, case):
    if case == "small":
        x, logits, experts, sh = _layer(pkg, dev, 1, 16, 16, 512, 256, 4)
        k = 4
    elif case == "one_expert":
        e, t = 8, 16
        logits = torch.full((t, e), -5.0, device=dev)
        logits[:, 3] = 5.0
        logits[:, 5] = 4.0
        x, logits, experts, sh = _layer(pkg, dev, 2, t, e, 512, 128, 2, shared=False, logits=logits)
        k = 2
    else:
        x, logits, experts, sh = _layer(pkg, dev, 3, 16, 256, 2048, 512, 8)
        k = 8
    layer = pkg.moe.MoEPlanLayer(experts, sh, tokens=x.shape[0], top_k=k)
    assert layer.shared_stacked == (sh is not None)
    y = layer(x, logits)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, k))
    # the per-launch path gives the same layer output (same math, only the
    # split of the K sums over CTAs differs)
    y2 = pkg.moe.moe_layer(x, logits, experts, sh, top_k=k)
    _assert_close(bf16_to_np_bits(y), bf16_to_np_bits(y2))
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_moe_plan_layer_reused_on_new_inputs(pkg, dev):
    """One plan, several calls with new tokens and new routing: every call
    matches the oracle (the route table and row buffers are rewritten in
    place before each run)."""
    x, logits, experts, sh = _layer(pkg, dev, 5, 16, 64, 1024, 256, 8)
    layer = pkg.moe.MoEPlanLayer(experts, sh, tokens=16, top_k=8)
    gen = torch.Generator(device=dev).manual_seed(6)
    for _ in range(3):
        x = torch.randn((16, 1024), generator=gen, device=dev).to(torch.bfloat16)
        logits = torch.randn((16, 64), generator=gen, device=dev)
        y = layer(x, logits)
        _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, 8))
    # a CUDA graph of the layer replays the same launches
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        layer(x, logits)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=s):
            yg = layer(x, logits)
    torch.cuda.current_stream(dev).wait_stream(s)
    x.copy_(torch.randn((16, 1024), generator=gen, device=dev).to(torch.bfloat16))
    logits.copy_(torch.randn((16, 64), generator=gen, device=dev))
    g.replay()
    torch.cuda.synchronize(dev)
    _assert_close(bf16_to_np_bits(yg), _oracle(x, logits, experts, sh, 8))
    del g
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0
