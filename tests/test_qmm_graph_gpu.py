"""Back-to-back launches in one CUDA graph sharing one workspace.

With programmatic dependent launch a launch starts while the previous one
(on the same stream, same workspace) is still finishing, so every access to
the split-K partial slots must wait for the previous launch.  A graph of
dense qmm launches (many split tiles), grouped MoE launches and the fused
gate/up + SiLU launch is replayed several times: every replay must equal the
eager results bit for bit and leave no device error.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import to_dev_bf16, to_dev_u32
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu


def test_graph_replays_match_eager(pkg, dev):
    import torch
    from dflash_mlx_b200 import _lib, moe as M

    rng = np.random.default_rng(3)
    dense = []
    for n, k in ((1024, 6144), (5120, 2048), (640, 17408), (2048, 1024)):
        w, s, b = oqmm.synth_weights(rng, n, k)
        dense.append((to_dev_u32(w, dev), to_dev_bf16(s, dev), to_dev_bf16(b, dev), k))
    xs = {k: to_dev_bf16(oqmm.synth_x(rng, 16, k), dev) for _, _, _, k in dense}
    wp = [(pkg.repack_pairs(w), s, b, k) for w, s, b, k in dense]
    gu_w, gu_s, gu_b = oqmm.synth_weights(rng, 1024, 2048)
    gu = (pkg.repack_pairs(to_dev_u32(gu_w, dev)), to_dev_bf16(gu_s, dev), to_dev_bf16(gu_b, dev))
    e, hid, inter = 64, 1024, 256

    def stack(n, k):
        q = torch.randint(-2**31, 2**31 - 1, (e, n, k // 8), dtype=torch.int64, device=dev).to(torch.int32)
        sc = (torch.rand((e, n, k // 64), device=dev) * 0.016 + 0.004)
        bi = (-8 * sc + torch.randn(sc.shape, device=dev) * 0.1 * sc)
        return M.QuantWeight(q, sc.to(torch.bfloat16), bi.to(torch.bfloat16))

    experts = {"gate": stack(inter, hid), "up": stack(inter, hid), "down": stack(hid, inter)}
    logits = torch.randn((16, e), device=dev)
    xm = torch.randn((16, hid), device=dev).to(torch.bfloat16)

    def body():
        outs = []
        for (w, s, b, k) in dense:
            outs.append(pkg.qmm_w4g64(xs[k], w, s, b))
        for (w, s, b, k) in wp:
            outs.append(pkg.qmm_w4g64(xs[k], w, s, b, layout="pairs"))
        outs.append(pkg.gate_up_silu(xs[2048], *gu))
        outs.append(M.moe_layer(xm, logits, experts, None, top_k=8))
        return outs

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        eager = [o.clone() for o in body()]
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            outs = body()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    for _ in range(6):
        graph.replay()
        torch.cuda.synchronize()
        for a, b in zip(outs, eager):
            assert torch.equal(a, b)
    assert _lib.device_error() == 0
