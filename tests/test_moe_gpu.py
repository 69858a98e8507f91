"""GPU parity of the MoE verify expert block (routing, grouped int4 qmm,
SiLU*up, weighted combine, shared expert) against the CPU oracle.

The reference has no test for this path (it is mlx-lm's SwitchGLU ->
mx.gather_qmm, not vendored): parity is against ``oracle/moe.py``'s
restatement, elementwise within |y - ref| <= 1e-2 + 2e-2 |ref| plus one
bf16 step of the row's largest output (2^-7 max_row |ref|: the rounding of
the intermediate projections, see _assert_close; bf16 out, fp32
accumulate).  Covered: a small configuration with ragged expert loads,
BASELINE config 2 (256 experts, top-8, hidden 2048, intermediate 512, one
shared expert, 16 tokens), the routing table itself, and a layer where one
expert takes every token (16 rows in one problem).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_to_np_bits, to_dev_bf16, to_dev_u32
from oracle import bf16 as obf16
from oracle import moe as omoe
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu


def _qweight(gen, dev, lead, n, k):
    """BASELINE weight distribution on the device (q ~ U{0..15}, s ~ U(0.004, 0.02),
    b = -8 s + N(0, 0.1 s))."""
    q = torch.randint(-2**31, 2**31 - 1, (*lead, n, k // 8), dtype=torch.int64, generator=gen,
                      device=dev).to(torch.int32)
    s = torch.rand((*lead, n, k // 64), generator=gen, device=dev) * 0.016 + 0.004
    b = -8 * s + torch.randn((*lead, n, k // 64), generator=gen, device=dev) * 0.1 * s
    return q, s.to(torch.bfloat16), b.to(torch.bfloat16)


def _np(t):
    if t.dtype == torch.bfloat16:
        return bf16_to_np_bits(t)
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    return t.cpu().numpy()


def _layer(pkg, dev, seed, t, e, h, inter, k, shared=True, logits=None):
    gen = torch.Generator(device=dev).manual_seed(seed)
    W = pkg.moe.QuantWeight
    experts = {name: W(*_qweight(gen, dev, (e,), n, kk))
               for name, n, kk in (("gate", inter, h), ("up", inter, h), ("down", h, inter))}
    sh = None
    if shared:
        sh = {name: W(*_qweight(gen, dev, (), n, kk))
              for name, n, kk in (("gate", inter, h), ("up", inter, h), ("down", h, inter))}
    x = torch.randn((t, h), generator=gen, device=dev).to(torch.bfloat16)
    if logits is None:
        logits = torch.randn((t, e), generator=gen, device=dev)
    return x, logits, experts, sh


def _oracle(x, logits, experts, sh, k):
    ids, _ = omoe.route_topk(logits.cpu().numpy(), k)
    used = np.unique(ids)
    oexp = {}
    for name in ("gate", "up", "down"):
        wq = experts[name]
        q, s, b = _np(wq.q), _np(wq.s), _np(wq.b)
        oexp[name + "_q"] = {int(i): q[i] for i in used}
        oexp[name + "_s"] = {int(i): s[i] for i in used}
        oexp[name + "_b"] = {int(i): b[i] for i in used}
    osh = None
    if sh is not None:
        osh = {}
        for name in ("gate", "up", "down"):
            osh[name + "_q"], osh[name + "_s"], osh[name + "_b"] = _np(sh[name].q), _np(sh[name].s), _np(sh[name].b)
    return omoe.moe_layer(_np(x), logits.cpu().numpy(), oexp, osh, top_k=k)


def _assert_close(y_bits, ref_bits):
    """Layer outputs: |y - ref| <= 1e-2 + 2e-2 |ref| + 2^-7 max_row |ref|.
    A layer output passes through two bf16-rounded projections and a
    weighted sum, so a one-step rounding difference in an intermediate
    (fp32 sums taken in another order) moves it by up to one bf16 step of
    the row's largest values, which the elementwise bound alone does not
    allow where outputs cancel to near zero.  A wrong expert, row or split-K
    partial moves outputs by their own magnitude and still fails."""
    y = obf16.to_f32(y_bits).astype(np.float64)
    r = obf16.to_f32(ref_bits).astype(np.float64)
    err = np.abs(y - r)
    row_scale = np.abs(r).max(axis=-1, keepdims=True)
    bad = err > 1e-2 + 2e-2 * np.abs(r) + 2.0 ** -7 * row_scale
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} outside tolerance, max err {err.max():.4g}"


def test_route_table(pkg, dev):
    gen = torch.Generator(device=dev).manual_seed(0)
    logits = torch.randn((16, 256), generator=gen, device=dev)
    table, w, ids = pkg.moe.route(logits, 8)
    ref_ids, ref_w = omoe.route_topk(logits.cpu().numpy(), 8)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    assert np.allclose(w.cpu().numpy(), ref_w, atol=1e-6)
    tb = table.cpu().numpy()
    p = tb[0]
    e = 256
    active = tb[1:1 + p]
    assert np.array_equal(active, np.unique(ref_ids))
    counts = tb[1 + e:1 + e + p]
    assert counts.sum() == 16 * 8
    for pi in range(p):
        toks = tb[1 + 2 * e + pi * 16: 1 + 2 * e + pi * 16 + counts[pi]]
        pairs = tb[1 + 18 * e + pi * 16: 1 + 18 * e + pi * 16 + counts[pi]]
        for tk, pr in zip(toks, pairs):
            assert pr // 8 == tk and ref_ids[tk, pr % 8] == active[pi]


def test_small_layer(pkg, dev):
    x, logits, experts, sh = _layer(pkg, dev, 1, 16, 16, 512, 256, 4)
    y = pkg.moe.moe_layer(x, logits, experts, sh, top_k=4)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, 4))


def test_one_expert_takes_all_tokens(pkg, dev):
    e, t = 8, 16
    logits = torch.full((t, e), -5.0, device=dev)
    logits[:, 3] = 5.0
    logits[:, 5] = 4.0
    x, logits, experts, sh = _layer(pkg, dev, 2, t, e, 512, 128, 2, shared=False, logits=logits)
    y = pkg.moe.moe_layer(x, logits, experts, None, top_k=2)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, None, 2))


def test_config2_baseline_layer(pkg, dev):
    x, logits, experts, sh = _layer(pkg, dev, 3, 16, 256, 2048, 512, 8)
    y = pkg.moe.moe_layer(x, logits, experts, sh, top_k=8)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, 8))
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0


def test_silu_mul_on_fused_gate_up_halves(pkg, dev):
    """Row-strided SiLU*up (halves of a fused gate|up output) equals the
    contiguous kernel and a float32 torch reference within one bf16 ulp."""
    import torch

    gen = torch.Generator(device=dev).manual_seed(3)
    gu = (torch.randn((16, 2 * 1000), generator=gen, device=dev) * 3).to(torch.bfloat16)
    g, u = gu[:, :1000], gu[:, 1000:]
    got = pkg.moe.silu_mul(g, u)
    assert got.is_contiguous() and got.shape == (16, 1000)
    same = pkg.moe.silu_mul(g.contiguous(), u.contiguous())
    assert torch.equal(got, same)
    ref = (torch.nn.functional.silu(g.float()) * u.float())
    assert torch.allclose(got.float(), ref, rtol=2 ** -7, atol=1e-6)


def test_fused_projection_equals_separate_launches(pkg, dev):
    """One launch over concatenated q|k|v weights gives the separate
    projections' results (same math, only the split-K partition differs)."""
    import torch

    rng = np.random.default_rng(9)
    parts = [oqmm.synth_weights(rng, n, 512) for n in (384, 128, 128)]
    x = oqmm.synth_x(rng, 16, 512)
    tx = to_dev_bf16(x, dev)
    fused = [np.concatenate([p[i] for p in parts], axis=0) for i in range(3)]
    y = pkg.qmm_w4g64(tx, to_dev_u32(fused[0], dev), to_dev_bf16(fused[1], dev),
                      to_dev_bf16(fused[2], dev))
    col = 0
    for w_q, s, b in parts:
        n = w_q.shape[0]
        ys = pkg.qmm_w4g64(tx, to_dev_u32(w_q, dev), to_dev_bf16(s, dev), to_dev_bf16(b, dev))
        a = y[:, col:col + n].float().cpu().numpy()
        e = ys.float().cpu().numpy()
        assert np.all(np.abs(a - e) <= 1e-2 + 2e-2 * np.abs(e))
        col += n


def _fused(pkg, experts, sh):
    from dflash_mlx_b200.verify_qmm import interleave_gate_up

    fe = {"gate_up": pkg.moe.fuse_expert_gate_up(experts["gate"], experts["up"]), "down": experts["down"]}
    fsh = None
    if sh is not None:
        W = pkg.moe.QuantWeight
        fsh = {"gate_up": W(interleave_gate_up(sh["gate"].q, sh["up"].q).contiguous(),
                            interleave_gate_up(sh["gate"].s, sh["up"].s).contiguous(),
                            interleave_gate_up(sh["gate"].b, sh["up"].b).contiguous()),
               "down": sh["down"]}
    return fe, fsh


@pytest.mark.parametrize("case", ["small", "config2"])
def test_fused_gate_up_silu_experts(pkg, dev, case):
    """Experts' gate/up interleaved and SiLU*up fused into the grouped launch
    (and the shared expert's into a dense launch): same layer output as the
    oracle, within the same tolerance."""
    if case == "small":
        x, logits, experts, sh = _layer(pkg, dev, 1, 16, 16, 512, 256, 4)
        k = 4
    else:
        x, logits, experts, sh = _layer(pkg, dev, 3, 16, 256, 2048, 512, 8)
        k = 8
    fe, fsh = _fused(pkg, experts, sh)
    y = pkg.moe.moe_layer(x, logits, fe, fsh, top_k=k)
    _assert_close(bf16_to_np_bits(y), _oracle(x, logits, experts, sh, k))
    from dflash_mlx_b200 import _lib
    assert _lib.device_error() == 0
