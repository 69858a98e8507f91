"""GPU parity of projection plans (tiled weights, one persistent launch).

* the tiled layout dequantises bit-exactly (one-hot activations read single
  weights back) with the subnormal and the general dequantiser;
* one-phase plans against the oracle (``oracle/qmm.py``, the reference's
  ``nib * s + b`` rounded to bf16, fp32 accumulation) on the benchmark's
  shapes, ragged N and K, 1..128 rows (every token tile: 16, 32, 64, 128),
  both dequantisers: elementwise ``|y - ref| <= 1e-2 + 2e-2 |ref|``; more
  than 128 rows as one phase per 128-row slice;
* the fused SiLU phase equals ``silu_mul`` of the plain phase bit for bit;
* a decoder layer as one plan (q|k|v, o, gate|up + SiLU, down reading the
  SiLU output through a dependency) equals the same phases run as separate
  plans bit for bit, and the oracle within tolerance;
* a chain where each phase reads the previous phase's output;
* repeated runs and CUDA-graph replays give identical bits and leave the
  workspace's counters zero.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import bf16_to_np_bits, to_dev_bf16, to_dev_u32
from oracle import bf16 as obf16
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 2e-2
COUNTER_BYTES = 64 * 1024   # a plan workspace's counter region (zero between runs)


def _assert_close(y_bits, ref_bits, what=""):
    yv = obf16.to_f32(y_bits).astype(np.float64)
    rv = obf16.to_f32(ref_bits).astype(np.float64)
    err = np.abs(yv - rv)
    bad = err > ATOL + RTOL * np.abs(rv)
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} outside tolerance, max err {err.max():.4g}"


def _tiled(pkg, dev, w_q, s, b, subnormal=None):
    return pkg.tile_weight(to_dev_u32(w_q, dev), to_dev_bf16(s, dev), to_dev_bf16(b, dev),
                           subnormal=subnormal)


@pytest.mark.parametrize("rows", [32, 128])
@pytest.mark.parametrize("subnormal", [True, False])
def test_tiled_dequant_is_exact(pkg, dev, subnormal, rows):
    # one-hot activations select single dequantised weights: y[m, n] = w[n, k_m]
    rng = np.random.default_rng(31)
    k, n = 1536, 320          # 3 K units, 3 tiles (the last one ragged)
    w_q, s, b = oqmm.synth_weights(rng, n, k)
    tw = _tiled(pkg, dev, w_q, s, b, subnormal=subnormal)
    assert tw.subnormal == subnormal
    w = oqmm.dequantize(w_q, s, b)
    for rep in range(2):
        cols = rng.choice(k, size=rows, replace=False)
        xf = np.zeros((rows, k), dtype=np.float32)
        xf[np.arange(rows), cols] = 1.0
        y = pkg.qmm_tiled(to_dev_bf16(obf16.from_f32(xf), dev), tw)
        assert np.array_equal(obf16.to_f32(bf16_to_np_bits(y)), w[:, cols].T)
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_subnormal_choice_follows_the_scales(pkg, dev):
    rng = np.random.default_rng(5)
    w_q, s, b = oqmm.synth_weights(rng, 128, 512)
    assert _tiled(pkg, dev, w_q, s, b).subnormal
    big = obf16.from_f32(np.full(s.shape, 0.05, np.float32))
    assert not _tiled(pkg, dev, w_q, big, b).subnormal


SHAPES = [
    ("config0", 16, 4096, 4096),
    ("qkv", 16, 5120, 8192),
    ("o", 16, 6144, 5120),
    ("down", 16, 17408, 5120),
    ("m1_tiny", 1, 64, 8),
    ("ragged", 17, 1600, 384),      # K % 512 != 0, N % 128 != 0, 32-row tile
    ("m32", 32, 5120, 1024),
    ("m5", 5, 640, 200),
    # several requests' rows in one token tile (64 / 128 rows: split-K
    # partials summed pass by pass, one or two accumulators)
    ("m48", 48, 5120, 1024),
    ("m64_qkv", 64, 5120, 8192),
    ("m100_ragged", 100, 1600, 384),
    ("m128_o", 128, 6144, 5120),
    ("m128_down", 128, 17408, 5120),
    # N % 8 != 0 at a 64-row tile: one store per value instead of 16-byte rows
    ("m40_n196", 40, 1024, 196),
]


@pytest.mark.parametrize("name,m,k,n", SHAPES)
@pytest.mark.parametrize("subnormal", [True, False])
def test_one_phase_matches_oracle(pkg, dev, name, m, k, n, subnormal):
    rng = np.random.default_rng(1000 + m * 7 + k + n)
    w_q, s, b = oqmm.synth_weights(rng, n, k)
    x = oqmm.synth_x(rng, m, k)
    y = pkg.qmm_tiled(to_dev_bf16(x, dev), _tiled(pkg, dev, w_q, s, b, subnormal=subnormal))
    _assert_close(bf16_to_np_bits(y), oqmm.qmm(x, w_q, s, b, accum=np.float32), name)


def test_reference_style_inputs_use_the_general_dequantiser(pkg, dev):
    # tests/test_verify_qmm_parity.py:44-53 inputs (x, w ~ N(0,1)/sqrt(K),
    # quantised): scales of N(0,1) weights exceed 2^-5, so the tiled layout
    # falls back to the general dequantiser; metric max_abs / (max|ref| + 1e-3)
    rng = np.random.default_rng(77)
    m, k, n = 16, 2048, 1024
    x = obf16.from_f32((rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32))
    w = obf16.round_f32(rng.standard_normal((n, k)).astype(np.float32))
    w_q, s, b = oqmm.affine_quantize(w)
    tw = _tiled(pkg, dev, w_q, s, b)
    assert not tw.subnormal
    y = bf16_to_np_bits(pkg.qmm_tiled(to_dev_bf16(x, dev), tw))
    max_abs, max_rel = oqmm.max_abs_rel(y, oqmm.qmm(x, w_q, s, b, accum=np.float32))
    assert max_rel <= 2e-2, (max_abs, max_rel)


def _gate_up(rng, inter, k):
    gq, gs, gb = oqmm.synth_weights(rng, inter, k)
    uq, us, ub = oqmm.synth_weights(rng, inter, k)

    def inter16(a, c):
        i = a.shape[0]
        return np.stack([a.reshape(i // 16, 16, -1), c.reshape(i // 16, 16, -1)], axis=1).reshape(2 * i, -1)

    return (gq, gs, gb), (uq, us, ub), (inter16(gq, uq), inter16(gs, us), inter16(gb, ub))


@pytest.mark.parametrize("m", [16, 32, 64, 128])
def test_silu_phase_equals_silu_of_plain_phase(pkg, dev, m):
    import torch

    rng = np.random.default_rng(9)
    inter, k = 1024, 2048
    g, u, gu = _gate_up(rng, inter, k)
    x = to_dev_bf16(oqmm.synth_x(rng, m, k), dev)
    tw = _tiled(pkg, dev, *gu)
    plain = pkg.qmm_tiled(x, tw)                       # [m, 2*inter] interleaved rows
    fused = pkg.qmm_tiled(x, tw, silu=True)            # [m, inter]
    pl = plain.view(m, inter // 16, 2, 16)
    ref = pkg.moe.silu_mul(pl[:, :, 0, :].reshape(m, inter).contiguous(),
                           pl[:, :, 1, :].reshape(m, inter).contiguous())
    assert torch.equal(fused, ref)


def _layer(pkg, dev, rng, hidden=1024, q_out=1536, kv=256, inter=2048, m=16):
    """Weights and buffers of a small decoder layer (four launches)."""
    import torch

    ws = {"qkv": oqmm.synth_weights(rng, q_out + 2 * kv, hidden),
          "o": oqmm.synth_weights(rng, hidden, q_out)}
    _, _, gu = _gate_up(rng, inter, hidden)
    ws["gate_up"] = gu
    ws["down"] = oqmm.synth_weights(rng, hidden, inter)
    tw = {k: _tiled(pkg, dev, *v) for k, v in ws.items()}
    x = to_dev_bf16(oqmm.synth_x(rng, m, hidden), dev)
    attn = to_dev_bf16(oqmm.synth_x(rng, m, q_out), dev)
    bufs = {"qkv": torch.empty((m, q_out + 2 * kv), dtype=torch.bfloat16, device=dev),
            "o": torch.empty((m, hidden), dtype=torch.bfloat16, device=dev),
            "h": torch.empty((m, inter), dtype=torch.bfloat16, device=dev),
            "down": torch.empty((m, hidden), dtype=torch.bfloat16, device=dev)}
    return ws, tw, x, attn, bufs


def _layer_phases(pkg, tw, x, attn, bufs, first=0):
    """The four phases of a layer starting at plan index ``first``, each
    waiting for the one before it (as in a forward pass, where attention and
    norms sit between the projections); down reads the SiLU output."""
    P = pkg.PlanPhase
    return [P(x, tw["qkv"], bufs["qkv"], dep=first - 1),
            P(attn, tw["o"], bufs["o"], dep=first),
            P(x, tw["gate_up"], bufs["h"], silu=True, dep=first + 1),
            P(bufs["h"], tw["down"], bufs["down"], dep=first + 2)]


@pytest.mark.parametrize("m", [16, 128])
def test_layer_plan_equals_separate_plans_and_oracle(pkg, dev, m):
    import torch

    rng = np.random.default_rng(12)
    ws, tw, x, attn, bufs = _layer(pkg, dev, rng, m=m)
    plan = pkg.ProjectionPlan(_layer_phases(pkg, tw, x, attn, bufs))
    plan.run()
    got = {k: v.clone() for k, v in bufs.items()}
    # each phase alone (its split over the SMs depends only on its own shape)
    sep_qkv = pkg.qmm_tiled(x, tw["qkv"])
    sep_o = pkg.qmm_tiled(attn, tw["o"])
    sep_h = pkg.qmm_tiled(x, tw["gate_up"], silu=True)
    sep_down = pkg.qmm_tiled(sep_h, tw["down"])
    for name, sep in (("qkv", sep_qkv), ("o", sep_o), ("h", sep_h), ("down", sep_down)):
        assert torch.equal(got[name], sep), name
    # oracle on the projections whose inputs are fixed
    xb, ab = bf16_to_np_bits(x), bf16_to_np_bits(attn)
    _assert_close(bf16_to_np_bits(got["qkv"]), oqmm.qmm(xb, *ws["qkv"], accum=np.float32), "qkv")
    _assert_close(bf16_to_np_bits(got["o"]), oqmm.qmm(ab, *ws["o"], accum=np.float32), "o")
    _assert_close(bf16_to_np_bits(got["down"]),
                  oqmm.qmm(bf16_to_np_bits(got["h"]), *ws["down"], accum=np.float32), "down")
    assert int(plan.workspace[:COUNTER_BYTES].count_nonzero()) == 0
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_rows_beyond_one_tile_run_as_slices(pkg, dev):
    """200 rows: two phases (128 + 72 rows) of one plan at the 128-row tile."""
    rng = np.random.default_rng(210)
    m, k, n = 200, 5120, 1024
    w_q, s, b = oqmm.synth_weights(rng, n, k)
    x = oqmm.synth_x(rng, m, k)
    y = pkg.qmm_tiled(to_dev_bf16(x, dev), _tiled(pkg, dev, w_q, s, b))
    _assert_close(bf16_to_np_bits(y), oqmm.qmm(x, w_q, s, b, accum=np.float32), "200 rows")


@pytest.mark.parametrize("dims", [[2048, 1024, 3072, 512, 2048],
                                  [1024, 1088, 704, 2048]])      # ragged tiles per 512-column group
def test_chain_reads_previous_outputs(pkg, dev, dims):
    """Phase i reads phase i-1's output; a result is only right if every
    phase waited for the whole of the previous one (ragged last tiles
    included)."""
    import torch

    rng = np.random.default_rng(44)
    tws, raw = [], []
    for i in range(len(dims) - 1):
        w_q, s, b = oqmm.synth_weights(rng, dims[i + 1], dims[i])
        s = obf16.from_f32(obf16.to_f32(s) * 0.25)   # keep activations O(1) along the chain
        raw.append((w_q, s, b))
        tws.append(_tiled(pkg, dev, w_q, s, b))
    x0 = to_dev_bf16(oqmm.synth_x(rng, 16, dims[0]), dev)
    outs = [torch.empty((16, d), dtype=torch.bfloat16, device=dev) for d in dims[1:]]
    ins = [x0] + outs[:-1]
    plan = pkg.ProjectionPlan([pkg.PlanPhase(ins[i], tws[i], outs[i], dep=i - 1)
                               for i in range(len(tws))])
    for _ in range(3):
        for o in outs:
            o.fill_(float("nan"))
        plan.run()
        torch.cuda.synchronize(dev)
        xb = bf16_to_np_bits(x0)
        for i, (w_q, s, b) in enumerate(raw):
            _assert_close(bf16_to_np_bits(outs[i]), oqmm.qmm(xb, w_q, s, b, accum=np.float32), f"link {i}")
            xb = bf16_to_np_bits(outs[i])
        assert int(plan.workspace[:COUNTER_BYTES].count_nonzero()) == 0


@pytest.mark.parametrize("m", [16, 128])
def test_down_waits_for_the_silu_columns_it_reads(pkg, dev, m):
    """gate|up + SiLU (1088 outputs: 17 tiles, the last one ragged) then
    down reading its output through a dependency: the SiLU output equals a
    one-phase plan's bit for bit and down matches the oracle, run twice."""
    import torch

    rng = np.random.default_rng(515)
    hidden, inter = 1024, 1088
    _, _, gu = _gate_up(rng, inter, hidden)
    down = oqmm.synth_weights(rng, hidden, inter)
    tgu, tdown = _tiled(pkg, dev, *gu), _tiled(pkg, dev, *down)
    x = oqmm.synth_x(rng, m, hidden)
    xd = to_dev_bf16(x, dev)
    h = torch.empty((m, inter), dtype=torch.bfloat16, device=dev)
    y = torch.empty((m, hidden), dtype=torch.bfloat16, device=dev)
    plan = pkg.ProjectionPlan([pkg.PlanPhase(xd, tgu, h, silu=True), pkg.PlanPhase(h, tdown, y, dep=0)])
    for _ in range(2):
        h.fill_(float("nan"))
        y.fill_(float("nan"))
        plan.run()
        torch.cuda.synchronize(dev)
        assert torch.equal(h, pkg.qmm_tiled(xd, tgu, silu=True))
        _assert_close(bf16_to_np_bits(y), oqmm.qmm(bf16_to_np_bits(h), *down, accum=np.float32), "down")
        assert int(plan.workspace[:COUNTER_BYTES].count_nonzero()) == 0


def test_plan_repeats_and_replays_in_a_cuda_graph(pkg, dev):
    import torch

    rng = np.random.default_rng(3)
    ws, tw, x, attn, bufs = _layer(pkg, dev, rng, hidden=2048, q_out=2048, kv=512, inter=4096)
    phases = [ph for i in range(3) for ph in _layer_phases(pkg, tw, x, attn, bufs, first=4 * i)]
    plan = pkg.ProjectionPlan(phases)        # the layer three times: 12 phases
    plan.run()
    torch.cuda.synchronize(dev)
    first = {k: v.clone() for k, v in bufs.items()}
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        plan.run()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            plan.run()
        for _ in range(3):
            for v in bufs.values():
                v.zero_()
            g.replay()
    torch.cuda.synchronize(dev)
    for k in bufs:
        assert torch.equal(bufs[k], first[k]), k
    assert int(plan.workspace[:COUNTER_BYTES].count_nonzero()) == 0
    del g
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_plan_rejects_bad_phases(pkg, dev):
    import torch

    rng = np.random.default_rng(1)
    w_q, s, b = oqmm.synth_weights(rng, 256, 512)
    tw = _tiled(pkg, dev, w_q, s, b)
    x = torch.zeros((16, 512), dtype=torch.bfloat16, device=dev)
    y = torch.zeros((16, 256), dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        pkg.ProjectionPlan([pkg.PlanPhase(x, tw, y, dep=0)])            # dep on itself
    with pytest.raises(ValueError):
        pkg.ProjectionPlan([pkg.PlanPhase(torch.zeros((129, 512), dtype=torch.bfloat16, device=dev),
                                          tw, torch.zeros((129, 256), dtype=torch.bfloat16, device=dev))])
    with pytest.raises(ValueError):
        pkg.ProjectionPlan([pkg.PlanPhase(x, tw, y[:, :128])])          # wrong output width
    with pytest.raises(ValueError):
        pkg.ProjectionPlan([pkg.PlanPhase(x, tw, y, silu=True)])        # SiLU output is N/2 wide


@pytest.mark.parametrize("rows", [16, 32])
def test_withheld_partial_times_out_and_the_plan_recovers(pkg, dev, rows):
    """Failure path of a plan, made on the host: CTA 1 is told to withhold its
    split-K partials (its range lies inside tile 0 of a 640-unit phase, so CTA
    0 must sum its partial) and every wait is bounded by 20 ms, at 16-row
    tiles (partials summed before the accumulator is read) and 32-row tiles
    (summed pass by pass).  CTA 0's wait runs out, the plan-wide abort word
    stops every CTA (the second phase's CTAs were waiting for the first phase
    to complete), the launch ends in well under a second with the device
    error word set and the time-out recorded (split-K partial, phase 0, CTA
    0).  After the workspace is zeroed, the same plan gives the oracle's
    results."""
    import time

    import torch

    from dflash_mlx_b200 import _lib

    rng = np.random.default_rng(66)
    w0 = oqmm.synth_weights(rng, 8192, 5120)
    w1 = oqmm.synth_weights(rng, 1024, 8192)
    tw0, tw1 = _tiled(pkg, dev, *w0), _tiled(pkg, dev, *w1)
    x = oqmm.synth_x(rng, rows, 5120)
    xd = to_dev_bf16(x, dev)
    y0 = torch.empty((rows, 8192), dtype=torch.bfloat16, device=dev)
    y1 = torch.empty((rows, 1024), dtype=torch.bfloat16, device=dev)
    plan = pkg.ProjectionPlan([pkg.PlanPhase(xd, tw0, y0), pkg.PlanPhase(y0, tw1, y1, dep=0)])
    torch.cuda.synchronize(dev)
    assert _lib.device_error() == 0
    plan.set_test_fault(skip_partial_cta=1, wait_limit_ns=20_000_000)
    t0 = time.perf_counter()
    plan.run()
    torch.cuda.synchronize(dev)
    assert time.perf_counter() - t0 < 5.0
    assert plan.last_timeout() == (3, 0, 0)
    assert _lib.device_error() == 1
    # normal runs again
    plan.set_test_fault(-1, 1_000_000_000)
    plan.reset_workspace()
    plan.run()
    torch.cuda.synchronize(dev)
    assert plan.last_timeout() == (0, 0, 0)
    assert _lib.device_error() == 0
    ref0 = oqmm.qmm(x, *w0, accum=np.float32)
    _assert_close(bf16_to_np_bits(y0), ref0, "phase 0 after recovery")
    _assert_close(bf16_to_np_bits(y1), oqmm.qmm(bf16_to_np_bits(y0), *w1, accum=np.float32),
                  "phase 1 after recovery")


def test_strided_output_rows(pkg, dev):
    """y rows with a stride that is not a multiple of 8 (a view into a wider
    buffer) at a 64-row tile: same values as a contiguous y, columns outside
    the view untouched."""
    import torch

    rng = np.random.default_rng(21)
    m, k, n = 48, 1024, 512
    w_q, s_, b_ = oqmm.synth_weights(rng, n, k)
    tw = _tiled(pkg, dev, w_q, s_, b_)
    x = to_dev_bf16(oqmm.synth_x(rng, m, k), dev)
    wide = torch.full((m, n + 4), 7.0, dtype=torch.bfloat16, device=dev)
    y = wide[:, 2:2 + n]
    pkg.ProjectionPlan([pkg.PlanPhase(x, tw, y)]).run()
    ref = pkg.qmm_tiled(x, tw)
    assert torch.equal(y, ref)
    assert torch.all(wide[:, :2] == 7.0) and torch.all(wide[:, 2 + n:] == 7.0)


def test_grouped_phases_at_32_rows(pkg, dev):
    """Grouped gate|up + SiLU and scattered down phases over a sorted route
    table of 32 tokens x top-2 of 8 experts (problems of up to 32 rows: a
    32-row token tile), with the shared expert as dense phases, then the
    combine: equals the MoE oracle."""
    import torch

    from oracle import moe as omoe
    from test_moe_gpu import _assert_close, _layer, _oracle

    t, e, h, inter, k = 32, 8, 512, 256, 2
    x, logits, experts, sh = _layer(pkg, dev, 7, t, e, h, inter, k)
    logits[:, 1] += 3.0          # expert 1 takes most tokens: a problem of > 16 rows
    ids_np, w_np = omoe.route_topk(logits.cpu().numpy(), k)
    counts = np.bincount(ids_np.reshape(-1), minlength=e)
    assert counts.max() > 16
    ids = torch.as_tensor(ids_np, device=dev)
    w = torch.as_tensor(w_np, device=dev)
    M = pkg.moe
    gu = M.fuse_expert_gate_up(experts["gate"], experts["up"])
    tgu = pkg.qmm_plan.tile_expert_stack(gu.q, gu.s, gu.b)
    tdn = pkg.qmm_plan.tile_expert_stack(experts["down"].q, experts["down"].s, experts["down"].b)
    from dflash_mlx_b200.verify_qmm import interleave_gate_up
    sgu = M.QuantWeight(interleave_gate_up(sh["gate"].q, sh["up"].q).contiguous(),
                        interleave_gate_up(sh["gate"].s, sh["up"].s).contiguous(),
                        interleave_gate_up(sh["gate"].b, sh["up"].b).contiguous())
    tsgu = pkg.qmm_plan.tile_weight(sgu.q, sgu.s, sgu.b)
    tsdn = pkg.qmm_plan.tile_weight(sh["down"].q, sh["down"].s, sh["down"].b)
    bf = dict(dtype=torch.bfloat16, device=dev)
    x_in = torch.empty((t, h), **bf)
    route, xs = M.sort_pairs(ids, x, e, x_copy=x_in)
    hs = torch.empty((t * k, inter), **bf)
    pair_out = torch.empty((t * k, h), **bf)
    hsh = torch.empty((t, inter), **bf)
    so = torch.empty((t, h), **bf)
    P = pkg.PlanPhase
    plan = pkg.ProjectionPlan([
        P(x_in, tsgu, hsh, silu=True),
        P(xs, tgu, hs, silu=True, route=route, problem_rows=32),
        P(hsh, tsdn, so, dep=0),
        P(hs, tdn, pair_out, dep=1, route=route, problem_rows=32, scatter=True)])
    plan.run()
    y = M.combine(pair_out, w, so)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, k))
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0
