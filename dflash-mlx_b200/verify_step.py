"""Synthetic target-verify step on B200 (the path the benchmark times).

One verify cycle of the reference's decode loop
(``dflash_mlx/engine/spec_epoch.py:2022-2106``) restricted to its hot path,
for ``requests`` independent requests of 16 verify tokens on this GPU:

1. the int4 g64 verify projections of every decoder layer at M = 16 per
   request (q, k, v, o, gate, up, down; ``verify_linear.py`` ->
   ``verify_qmm.py``), with SiLU * up feeding down.  Projections that read
   the same input are stored concatenated (q|k|v, gate|up) and run as one
   launch each, 4 launches per layer; with several requests on the GPU two
   requests' rows share each launch (32 rows), so weights are read once per
   pair of requests;
2. the lm_head argmax + greedy acceptance epilogue (``spec_epoch.py:2067-2072``)
   on a vocabulary shard, keys all-gathered across ranks when the vocabulary
   is split;
3. GatedDeltaNet tape-replay rollback of every GDN layer with the accepted
   step counts straight from step 2 (``recurrent_rollback_cache.py:142-165``:
   ``accepted + 1`` steps), so no value is read back to the host; all layers'
   states share one arena and roll back in one launch.

Weights are random: nibbles uniform, scales ~ U(0.004, 0.02), biases
-8 * scale + N(0, 0.1 * scale) (no checkpoints offline).
The per-request qmm stack runs the same x through every layer (no attention
or residual stream: those are outside the hot path).  Each device-side part
is captured once in a CUDA graph and replayed; NCCL collectives (vocabulary
split across ranks) run between the graphs.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import lm_head as _lm
from .kernels import gated_delta_kernel_with_tape, tape_replay_
from .moe import QuantWeight, silu_mul
from .qmm_plan import MAX_ROWS, PlanPhase, ProjectionPlan, tile_weight
from .verify_qmm import gate_up_silu, qmm_w4g64, repack_pairs


def init_process_group(backend: str, *, timeout_s: float = 120.0, device=None):
    """``torch.distributed`` start-up for one rank of the step (rank, world
    size and rendezvous from RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT),
    bounded by ``timeout_s``: a rendezvous that cannot complete, or a
    collective whose peer is gone, ends with an exception after that long
    instead of waiting for ever.  Returns the default group."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    kw = {"device_id": device} if device is not None else {}
    try:
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=timedelta(seconds=timeout_s), **kw)
    except Exception as e:  # noqa: BLE001 - re-raised with the rendezvous named
        where = f"{os.environ.get('MASTER_ADDR', '?')}:{os.environ.get('MASTER_PORT', '?')}"
        raise RuntimeError(f"rank {rank}/{world}: {backend} process group at {where} did not start "
                           f"within {timeout_s:g} s: {e}") from e
    return dist.group.WORLD


@dataclass
class StackShape:
    hidden: int = 5120
    layers: int = 64
    q_out: int = 6144
    kv_out: int = 1024
    inter: int = 17408
    vocab: int = 248320
    gdn_layers: int = 48
    gdn_heads: int = 48
    gdn_dk: int = 128
    gdn_dv: int = 128
    block: int = 16

    def projections(self):
        """(name, out_features N, in_features K) of one decoder layer."""
        h = self.hidden
        return [("q", self.q_out, h), ("k", self.kv_out, h), ("v", self.kv_out, h),
                ("o", h, self.q_out), ("gate", self.inter, h), ("up", self.inter, h),
                ("down", h, self.inter)]

    def launches(self):
        """(name, N, K) of the qmm launches of one layer.  Projections that
        read the same input are stored concatenated along N, as fused-
        projection checkpoints do (q|k|v, gate|up), and run as one launch."""
        h = self.hidden
        return [("qkv", self.q_out + 2 * self.kv_out, h), ("o", h, self.q_out),
                ("gate_up", 2 * self.inter, h), ("down", h, self.inter)]

    def qmm_bytes_per_step(self, requests: int, per_launch: int = 1, silu_fused: bool = False) -> int:
        """Algorithmic bytes of the projection stack for ``requests`` requests on
        one GPU: weights (+ scales, biases) once per group of ``per_launch``
        requests whose rows share each launch or plan phase (2 for the
        per-call kernel's 32-row tile, 8 for the plan kernel's 128-row tile),
        and each request's activations."""
        launches = (requests + per_launch - 1) // per_launch
        total = 0
        for name, n, k in self.launches():
            n_out = n // 2 if (silu_fused and name == "gate_up") else n
            total += launches * (n * k // 2 + 2 * 2 * n * (k // 64)) + requests * 2 * self.block * (k + n_out)
        return total * self.layers

    def qmm_bytes_per_request(self, silu_fused: bool = False) -> int:
        """Algorithmic bytes of one request's projection stack: packed weights +
        bf16 scales and biases + bf16 activations in and out, per launch (the
        fused gate|up launch writes silu(gate) * up: half its rows)."""
        total = 0
        for name, n, k in self.launches():
            n_out = n // 2 if (silu_fused and name == "gate_up") else n
            total += n * k // 2 + 2 * 2 * n * (k // 64) + 2 * self.block * (k + n_out)
        return total * self.layers

    def qmm_flops_per_request(self) -> int:
        """Multiply-add FLOPs of one request's projection stack (16 rows)."""
        return 2 * self.block * sum(n * k for _, n, k in self.projections()) * self.layers


def _quant_weight(gen, dev, n, k):
    q = torch.randint(-2**31, 2**31 - 1, (n, k // 8), dtype=torch.int64, generator=gen,
                      device=dev).to(torch.int32)
    s = torch.rand((n, k // 64), generator=gen, device=dev) * 0.016 + 0.004
    b = -8 * s + torch.randn((n, k // 64), generator=gen, device=dev) * 0.1 * s
    return QuantWeight(q, s.to(torch.bfloat16), b.to(torch.bfloat16))


class VerifyStep:
    """Owns the synthetic weights and state of one GPU and runs verify steps."""

    def __init__(self, device: torch.device, *, requests: int = 1, shape: Optional[StackShape] = None,
                 rank: int = 0, world: int = 1, group=None, seed: int = 0,
                 weight_layout: str = "mlx", fuse_silu: bool = False, pack_requests: bool = True,
                 qmm_deps: str = "dataflow", share_weights: Optional["VerifyStep"] = None,
                 collectives_in_graph: bool = True):
        """``share_weights``: another step on the same device, rank and shape
        whose decoder and lm_head weights this one reuses (a different number
        of requests over the same model).  ``collectives_in_graph``: with
        several ranks, capture the all-gathers of the vocabulary-split lm_head
        in the same CUDA graph as the keys, acceptance and rollback (False:
        issue them from the host between graphs)."""
        self.dev = torch.device(device)
        if weight_layout not in ("mlx", "pairs", "tiled"):
            raise ValueError(f"unknown weight layout {weight_layout!r}")
        self.weight_layout = weight_layout
        if fuse_silu and weight_layout == "mlx":
            raise ValueError("the fused SiLU epilogue takes pair-packed or tiled weights")
        if weight_layout == "tiled" and not fuse_silu:
            raise ValueError("the tiled (plan) stack runs gate|up with the fused SiLU epilogue")
        # fuse_silu: the gate|up weights are read as the gate and up rows
        # interleaved in blocks of 16 (interleave_gate_up) and one launch
        # writes silu(gate) * up
        self.fuse_silu = bool(fuse_silu)
        self.pack_requests = bool(pack_requests)
        # requests whose rows share one read of every weight
        self.requests_per_launch = (MAX_ROWS // (shape or StackShape()).block if weight_layout == "tiled"
                                    else 2 if self.pack_requests else 1)
        self.shape = shape or StackShape()
        self.requests = int(requests)
        self.rank, self.world, self.group = rank, world, group
        sh = self.shape
        if share_weights is not None:
            o = share_weights
            if (o.dev != self.dev or o.shape != sh or o.weight_layout != weight_layout or o.rank != rank
                    or o.world != world):
                raise ValueError("share_weights needs a step on the same device, shape, layout and rank")
            self.layers, self.tiled = o.layers, getattr(o, "tiled", None)
        else:
            gen = torch.Generator(device=self.dev).manual_seed(seed)
            # replicated decoder weights (identical on every rank: same seed), in
            # the fused launch layout (q|k|v and gate|up concatenated along N)
            self.layers = [{name: _quant_weight(gen, self.dev, n, k) for name, n, k in sh.launches()}
                           for _ in range(sh.layers)]
        if share_weights is not None:
            pass
        elif weight_layout == "pairs":
            # load-time repack into the pair-packed nibble order (in place)
            for lw in self.layers:
                for qw in lw.values():
                    repack_pairs(qw.q, out=qw.q)
        elif weight_layout == "tiled":
            # load-time repack into the plan kernel's tiled layout; the MLX-packed
            # copies are dropped once tiled
            tiled = []
            for lw in self.layers:
                tiled.append({name: tile_weight(qw.q, qw.s, qw.b) for name, qw in lw.items()})
                lw.clear()
            self.tiled = tiled
            self.layers = None
        # this rank's vocabulary shard of the bf16 lm_head, N(0, 0.02)
        self.v_begin, v_len = _lm.vocab_shard(sh.vocab, rank, world)
        if share_weights is not None:
            self.lm_w = share_weights.lm_w
        else:
            wgen = torch.Generator(device=self.dev).manual_seed(seed + 1000 + rank)
            self.lm_w = (torch.randn((v_len, sh.hidden), generator=wgen, device=self.dev) * 0.02).to(torch.bfloat16)
        # GDN rollback snapshot states [layer, B, Hv, Dv, Dk] fp32 ~ N(0, 0.05)
        # and the tapes of one verify block, recorded by the verify forward
        # (gated_delta_kernel_with_tape) from synthetic inputs:
        # q, k, v bf16 ~ N(0, 1) (q, k L2-normalised), beta = sigmoid(N),
        # g = exp(-softplus(N)).
        b, t, hv, dk, dv = self.requests, sh.block, sh.gdn_heads, sh.gdn_dk, sh.gdn_dv
        sgen = torch.Generator(device=self.dev).manual_seed(seed + 2000 + rank)
        self.gdn_state = torch.randn((sh.gdn_layers, b, hv, dv, dk), generator=sgen, device=self.dev) * 0.05

        def _unit(shape):
            a = torch.randn(shape, generator=sgen, device=self.dev)
            return (a / a.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

        self.tape_k = _unit((sh.gdn_layers, b, t, hv, dk))
        self.tape_g = torch.exp(-torch.nn.functional.softplus(
            torch.randn((sh.gdn_layers, b, t, hv), generator=sgen, device=self.dev)))
        self.tape = torch.empty((sh.gdn_layers, b, t, hv, dv), device=self.dev)
        for layer in range(sh.gdn_layers):
            q = _unit((b, t, hv, dk))
            v = torch.randn((b, t, hv, dv), generator=sgen, device=self.dev).to(torch.bfloat16)
            beta = torch.sigmoid(torch.randn((b, t, hv), generator=sgen, device=self.dev))
            _, _, self.tape[layer] = gated_delta_kernel_with_tape(
                q, self.tape_k[layer], v, self.tape_g[layer], beta, self.gdn_state[layer])
        # step inputs / outputs (static buffers for graph replay)
        self.x = torch.empty((b * sh.block, sh.hidden), dtype=torch.bfloat16, device=self.dev)
        # stand-in for the attention output feeding o_proj (produced outside
        # the verify hot path; fixed random rows)
        self.attn_out = (torch.randn((b * sh.block, sh.q_out), generator=sgen, device=self.dev)
                         * 0.5).to(torch.bfloat16)
        self.verify_ids = torch.zeros((b, sh.block), dtype=torch.int32, device=self.dev)
        self.stream = torch.cuda.Stream(self.dev)
        self.graphs = None
        self.ev = None
        self.qmm_deps = qmm_deps
        self.collectives_in_graph = collectives_in_graph
        self.plan = self._build_plan(qmm_deps) if weight_layout == "tiled" else None

    def _build_plan(self, deps: str = "dataflow") -> ProjectionPlan:
        """The whole projection stack as one plan, requests in groups of up to
        eight (128 rows per phase: one token tile, so the group's requests
        share one read of every weight).  Every layer writes its own output
        buffers.

        ``deps="dataflow"``: a projection waits on the device for exactly the
        projections whose outputs it reads -- down for gate|up's SiLU output,
        and the next layer's q|k|v for this layer's down output (its input).
        o and gate|up read fixed stand-ins for the attention output and the
        normalised residual, which ops outside this path produce.
        ``deps="chain"``: every projection also waits for the one before it
        (q|k|v -> o -> gate|up -> down -> next q|k|v), as when attention and
        norms run between them in the same launch order."""
        if deps not in ("dataflow", "chain"):
            raise ValueError(f"unknown dependency mode {deps!r}")
        sh = self.shape
        rows = self.requests * sh.block
        groups = [(g0, min(rows, g0 + MAX_ROWS)) for g0 in range(0, rows, MAX_ROWS)]

        def buf(m, n):
            return torch.empty((m, n), dtype=torch.bfloat16, device=self.dev)

        outs = []
        phases = []
        last_down = [None] * len(groups)      # (phase index, tensor) of each group's last down
        chain = deps == "chain"
        for lt in self.tiled:
            # projection-major inside a layer (every group's q|k|v, then every
            # o, gate|up, down), so with several groups a projection's input
            # was written a few phases earlier and its wait is short
            layer_out = [{"qkv": buf(g1 - g0, sh.q_out + 2 * sh.kv_out), "o": buf(g1 - g0, sh.hidden),
                          "h": buf(g1 - g0, sh.inter), "down": buf(g1 - g0, sh.hidden)}
                         for g0, g1 in groups]
            idx = {}
            for gi, (g0, g1) in enumerate(groups):
                prev = last_down[gi]
                x_in = self.x[g0:g1] if prev is None else prev[1]
                idx["qkv", gi] = len(phases)
                phases.append(PlanPhase(x_in, lt["qkv"], layer_out[gi]["qkv"],
                                        dep=-1 if prev is None else prev[0]))
            for gi, (g0, g1) in enumerate(groups):
                idx["o", gi] = len(phases)
                phases.append(PlanPhase(self.attn_out[g0:g1], lt["o"], layer_out[gi]["o"],
                                        dep=idx["qkv", gi] if chain else -1))
            for gi, (g0, g1) in enumerate(groups):
                idx["gate_up", gi] = len(phases)
                phases.append(PlanPhase(self.x[g0:g1], lt["gate_up"], layer_out[gi]["h"], silu=True,
                                        dep=idx["o", gi] if chain else -1))
            for gi in range(len(groups)):
                idx["down", gi] = len(phases)
                phases.append(PlanPhase(layer_out[gi]["h"], lt["down"], layer_out[gi]["down"],
                                        dep=idx["gate_up", gi]))
                last_down[gi] = (idx["down", gi], layer_out[gi]["down"])
            outs.append(layer_out)
        self.plan_out = outs
        self.last_qkv = outs[-1][0]["qkv"]
        self.last_down = outs[-1][0]["down"]
        return ProjectionPlan(phases)

    # -------------------------------------------------------------- parts
    def _qmm_stack(self):
        if self.plan is not None:
            self.plan.run()
            return
        sh = self.shape
        # With several requests on this GPU their rows go through each launch
        # together: the qmm takes up to 32 rows per launch (two requests'
        # 16-token blocks), so each weight is read once per pair of requests.
        groups = [(0, self.requests)] if self.pack_requests else [(r, r + 1) for r in range(self.requests)]
        for r0, r1 in groups:
            x = self.x[r0 * sh.block:r1 * sh.block]
            a = self.attn_out[r0 * sh.block:r1 * sh.block]
            lay = self.weight_layout
            for lw in self.layers:
                self.last_qkv = qmm_w4g64(x, lw["qkv"].q, lw["qkv"].s, lw["qkv"].b, layout=lay)
                qmm_w4g64(a, lw["o"].q, lw["o"].s, lw["o"].b, layout=lay)
                if self.fuse_silu:
                    h = gate_up_silu(x, lw["gate_up"].q, lw["gate_up"].s, lw["gate_up"].b)
                else:
                    gu = qmm_w4g64(x, lw["gate_up"].q, lw["gate_up"].s, lw["gate_up"].b, layout=lay)
                    h = silu_mul(gu[:, :sh.inter], gu[:, sh.inter:])
                self.last_down = qmm_w4g64(h, lw["down"].q, lw["down"].s, lw["down"].b, layout=lay)

    def _keys(self, hidden_all):
        self.keys = _lm.lm_head_argmax_keys(hidden_all, self.lm_w, v_begin=self.v_begin)

    def _accept_and_rollback(self, keys_all, ids_all):
        post, acc, nxt, _ = _lm.verify_accept(keys_all, ids_all, block=self.shape.block)
        b0 = self.rank * self.requests
        self.posterior = post[b0:b0 + self.requests]
        self.acceptance = acc[b0:b0 + self.requests]
        self.next_token = nxt[b0:b0 + self.requests]
        steps = self.acceptance + 1       # recurrent_rollback_cache.py:154
        # The GDN states of all layers live in one [L, B, Hv, Dv, Dk] arena, so
        # the rollback of every layer is a single launch with the layer folded
        # into the batch (sequence i of layer l is batch entry l * B + i).
        sh = self.shape
        lb = sh.gdn_layers * self.requests
        tape_replay_(self.gdn_state.view(lb, *self.gdn_state.shape[2:]),
                     self.tape.view(lb, *self.tape.shape[2:]),
                     self.tape_k.view(lb, *self.tape_k.shape[2:]),
                     self.tape_g.view(lb, *self.tape_g.shape[2:]),
                     steps.repeat(sh.gdn_layers))

    def _exchange(self, with_collectives: bool = True):
        """lm_head keys and acceptance + rollback; with several ranks the
        hidden rows and verify ids are all-gathered before the keys and the
        8-byte row keys after them (vocabulary split)."""
        if self.world > 1:
            import torch.distributed as dist

            if with_collectives:
                dist.all_gather_into_tensor(self.x_all, self.x, group=self.group)
                dist.all_gather_into_tensor(self.ids_all, self.verify_ids, group=self.group)
            self._keys(self.x_all)
            if with_collectives:
                dist.all_gather_into_tensor(self.keys_all.view(-1), self.keys, group=self.group)
        else:
            self._keys(self.x_all)
            self.keys_all.view(-1).copy_(self.keys)
        self._accept_and_rollback(self.keys_all, self.ids_all)

    # -------------------------------------------------------------- driving
    def capture(self):
        """Warm up once eagerly, then capture the device parts in CUDA graphs:
        A = qmm stack, B = lm_head keys + acceptance + rollback, with the
        all-gathers of several ranks inside B (``collectives_in_graph``; the
        eager warm-up creates the communicator first) or issued from the host
        between the lm_head keys and the rest."""
        sh = self.shape
        rows = self.requests * sh.block
        with torch.cuda.device(self.dev), torch.cuda.stream(self.stream):
            if self.world == 1:
                self.x_all, self.ids_all = self.x, self.verify_ids
            else:
                self.x_all = torch.empty((self.world * rows, sh.hidden), dtype=torch.bfloat16,
                                         device=self.dev)
                self.ids_all = torch.empty((self.world * self.requests, sh.block), dtype=torch.int32,
                                           device=self.dev)
            self.keys_all = torch.empty((self.world, self.world * rows), dtype=torch.int64,
                                        device=self.dev)
            self._qmm_stack()
            in_graph = self.world == 1 or self.collectives_in_graph
            self._exchange(with_collectives=in_graph)
            self.stream.synchronize()
            ga = torch.cuda.CUDAGraph()
            with torch.cuda.graph(ga, stream=self.stream):
                self._qmm_stack()
            if in_graph:
                gb = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gb, stream=self.stream):
                    self._exchange()
                self.graphs = [ga, gb]
            else:
                gb, gc = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                with torch.cuda.graph(gb, stream=self.stream):
                    self._keys(self.x_all)
                with torch.cuda.graph(gc, stream=self.stream):
                    self._accept_and_rollback(self.keys_all, self.ids_all)
                self.graphs = [ga, gb, gc]
        torch.cuda.synchronize(self.dev)

    def run_step(self, ev_qmm: Optional[tuple] = None):
        """One verify step on self.stream (graphs must be captured).  With
        ``ev_qmm = (start, end)`` the qmm stack is bracketed by those events."""
        with torch.cuda.device(self.dev), torch.cuda.stream(self.stream):
            if ev_qmm is not None:
                ev_qmm[0].record(self.stream)
            self.graphs[0].replay()
            if ev_qmm is not None:
                ev_qmm[1].record(self.stream)
            if len(self.graphs) == 2:
                self.graphs[1].replay()
            else:
                # several ranks, collectives issued from the host between graphs
                import torch.distributed as dist

                dist.all_gather_into_tensor(self.x_all, self.x, group=self.group)
                dist.all_gather_into_tensor(self.ids_all, self.verify_ids, group=self.group)
                self.graphs[1].replay()
                dist.all_gather_into_tensor(self.keys_all.view(-1), self.keys, group=self.group)
                self.graphs[2].replay()

    def verify(self, x_host: torch.Tensor, verify_ids_host: torch.Tensor):
        """End-to-end call: copy this rank's inputs from (pinned) host memory,
        run one step, return (posterior, acceptance, next_token) on the host."""
        with torch.cuda.stream(self.stream):
            self.x.copy_(x_host, non_blocking=True)
            self.verify_ids.copy_(verify_ids_host, non_blocking=True)
        self.run_step()
        with torch.cuda.stream(self.stream):
            out = torch.cat([self.posterior.reshape(-1), self.acceptance, self.next_token]).to(
                "cpu", non_blocking=True)
        self.stream.synchronize()
        return out
