"""Oracle for the MoE verify ``gather_qmm`` expert path -- TEST INFRASTRUCTURE ONLY.

The reference reaches routed experts through mlx-lm's ``SwitchGLU`` /
``SwitchLinear`` -> ``mx.gather_qmm`` (third party: mlx >= 0.31.0 and
mlx-lm >= 0.31.0, pinned in the reference's ``pyproject.toml:14-17``; neither
is vendored), called from the decoder layers at
``dflash_mlx/engine/target_qwen_gdn.py:863-865``.  This restates the published
algorithm of that block for one layer:

1. router: softmax over all experts, keep the top-k, renormalise the kept
   probabilities (identical to a softmax over the top-k logits);
2. for every (token, slot) pair with expert e:
   ``h = silu(x @ Wg_e.T) * (x @ Wu_e.T)`` and ``o = h @ Wd_e.T``, each matmul an
   affine int4 g64 qmm (``oracle/qmm.py``) whose output is rounded to bf16;
3. ``y_t = sum_j score[t, j] * o[t, j]`` in fp32 (slot order j = 0..k-1), plus
   the shared expert's output, rounded to bf16.

MLX/MoE parity is **unpinned**: no reference test exercises this path.
"""

from __future__ import annotations

import numpy as np

from . import bf16
from .qmm import dequantize


def route_topk(logits: np.ndarray, k: int):
    """Top-k experts per token and their renormalised softmax weights.

    Ordering: descending logit, ties to the lower expert id.
    Returns (ids int32 [T, k], weights float32 [T, k]).
    """
    lg = np.asarray(logits, dtype=np.float32)
    t, e = lg.shape
    order = np.lexsort((np.broadcast_to(np.arange(e), lg.shape), -lg), axis=-1)
    ids = order[:, :k].astype(np.int32)
    top = np.take_along_axis(lg, ids.astype(np.int64), axis=-1).astype(np.float64)
    w = np.exp(top - top.max(axis=-1, keepdims=True))
    w = w / w.sum(axis=-1, keepdims=True)
    return ids, w.astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return x / (1.0 + np.exp(-x))


def _mm(xf: np.ndarray, w: np.ndarray) -> np.ndarray:
    return bf16.round_f32((xf.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32))


def expert_mlp(xf, wg, sg, bg, wu, su, bu, wd, sd, bd):
    """One expert on bf16-valued float32 rows ``xf`` -> bf16-valued float32 output."""
    g = _mm(xf, dequantize(wg, sg, bg))
    u = _mm(xf, dequantize(wu, su, bu))
    h = bf16.round_f32(silu(g) * u)
    return _mm(h, dequantize(wd, sd, bd))


def moe_layer(x, router_logits, experts, shared, top_k: int = 8):
    """One MoE layer.

    ``x`` bf16 bits ``[T, H]``; ``experts`` is a dict with uint32 / bf16-bit arrays
    ``gate_q [E, I, H/8]``, ``gate_s``/``gate_b [E, I, H/64]``, ``up_*`` alike,
    ``down_q [E, H, I/8]``, ``down_s``/``down_b [E, H, I/64]``; ``shared`` has the
    same keys without the expert axis (or is None).  Returns bf16 bits ``[T, H]``.
    """
    xf = bf16.to_f32(x)
    t, hdim = xf.shape
    ids, w = route_topk(router_logits, top_k)
    y = np.zeros((t, hdim), dtype=np.float32)
    cache = {}
    for e in np.unique(ids):
        cache[int(e)] = None
    outs = np.zeros((t, top_k, hdim), dtype=np.float32)
    for e in cache:
        rows, slots = np.nonzero(ids == e)
        o = expert_mlp(xf[rows],
                       experts["gate_q"][e], experts["gate_s"][e], experts["gate_b"][e],
                       experts["up_q"][e], experts["up_s"][e], experts["up_b"][e],
                       experts["down_q"][e], experts["down_s"][e], experts["down_b"][e])
        outs[rows, slots] = o
    for j in range(top_k):
        y = (y + w[:, j:j + 1] * outs[:, j]).astype(np.float32)
    if shared is not None:
        so = expert_mlp(xf, shared["gate_q"], shared["gate_s"], shared["gate_b"],
                        shared["up_q"], shared["up_s"], shared["up_b"],
                        shared["down_q"], shared["down_s"], shared["down_b"])
        y = (y + so).astype(np.float32)
    return bf16.from_f32(y)


def distinct_experts(router_logits, top_k: int = 8) -> int:
    ids, _ = route_topk(router_logits, top_k)
    return int(np.unique(ids).size)
