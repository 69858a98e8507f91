"""Benchmark of the dflash-mlx target-verify hot path on B200.

One step = one synthetic verify cycle per request (BASELINE configs 1 + 3 + 4):
the 64-layer int4 g64 verify projection stack at M = 16 tokens per request
(hidden 5120: q 5120->6144, k/v 5120->1024, o 6144->5120, gate/up
5120->17408, down 17408->5120; same-input projections stored concatenated and
run as one launch each: q|k|v, o, gate|up, down), the lm_head (248320 x 5120 bf16) argmax +
greedy acceptance of 16 verify ids, and the GatedDeltaNet tape-replay
rollback of 48 layers (48 heads, 128 x 128 fp32 state) with the accepted
step counts.  Requests are data-parallel across GPUs (weak scaling:
``--requests-per-gpu`` per rank); the lm_head vocabulary is split across
ranks and the per-row argmax keys are all-gathered over NCCL.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``
prints one JSON line (rank 0).  ``--impl reference`` times the reference's
algorithm on the host cores (the CPU restatement in ``oracle/``; MLX cannot
run here) on a bounded sample of the same step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "verify-steps/s: 64-layer int4 g64 verify qmm stack (M=16) + lm_head argmax/accept + 48-layer GDN rollback"
UNIT = "verify-steps/s"


def _peaks():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic_per_launch():
    """DRAM bytes per qmm launch (mean over the four launch kinds of a layer)
    from the committed ncu summary, if present."""
    f = ROOT / "profiles" / "qmm_w4g64_verify_layer_launches.md"
    try:
        for line in f.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                return int(line.split(":")[1].strip()), line
    except Exception:
        pass
    return None, None


# ------------------------------------------------------------------ CPU arm
def cpu_step_sample(scale_layers: bool = True):
    """Time the reference algorithm (oracle restatement) on a bounded sample of
    one step and scale it to the full step.  Returns (seconds per step, sample text)."""
    import numpy as np

    from oracle import gdn as ogdn
    from oracle import lmhead as olm
    from oracle import qmm as oqmm

    rng = np.random.default_rng(0)
    x = oqmm.synth_x(rng, 16, 5120)
    t_qmm = 0.0
    # sample: the q projection of one layer (31.5 M weights) -> scale by the
    # stack's weight count
    w_q, s, b = oqmm.synth_weights(rng, 6144, 5120)
    t0 = time.perf_counter()
    oqmm.qmm(x, w_q, s, b, accum=np.float32)
    t_q = time.perf_counter() - t0
    stack_weights = 64 * (6144 * 5120 + 2 * 1024 * 5120 + 5120 * 6144 + 2 * 17408 * 5120 + 5120 * 17408)
    t_qmm = t_q * stack_weights / (6144 * 5120)
    # lm_head: 16 rows against a 1/64 vocabulary slice, scaled by 64
    h = oqmm.synth_x(rng, 16, 5120)
    from oracle import bf16 as obf16
    w = obf16.from_f32((rng.standard_normal((248320 // 64, 5120)) * 0.02).astype(np.float32))
    t0 = time.perf_counter()
    lg = olm.logits_bf16(h, w)
    post = olm.greedy_tokens(lg).reshape(1, 16)
    ids = olm.synth_verify_ids(rng, post, 248320)
    olm.verify_accept(lg.reshape(1, 16, -1), ids)
    t_lm = (time.perf_counter() - t0) * 64
    # GDN: one layer of 48 heads, 16 recorded steps, scaled by 48 layers
    st = (rng.standard_normal((1, 48, 128, 128)) * 0.05).astype(np.float32)
    kk = rng.standard_normal((1, 16, 48, 128)).astype(np.float32)
    tape = rng.standard_normal((1, 16, 48, 128)).astype(np.float32)
    g = rng.random((1, 16, 48)).astype(np.float32)
    t0 = time.perf_counter()
    ogdn.tape_replay_accepted(tape, kk, g, st, np.array([9]))
    t_gdn = (time.perf_counter() - t0) * 48
    total = t_qmm + t_lm + t_gdn
    sample = ("q projection 6144x5120 of one layer (scaled x%.1f to the 64-layer stack), lm_head "
              "16 rows x 3880 vocab (x64), GDN replay 1 layer 48 heads (x48); numpy, %d host threads"
              % (stack_weights / (6144 * 5120), os.cpu_count()))
    return total, sample, {"qmm_s": t_qmm, "lm_head_s": t_lm, "gdn_s": t_gdn}


def workload_name(layers: int = 64) -> str:
    """The verify-step workload both arms time (config.workload)."""
    return (f"verify step = config1 ({layers}-layer int4 g64 qmm stack, hidden 5120, "
            "M=16 per request) + config3 (lm_head 248320x5120 bf16, vocab split over "
            "ranks) + config4 (48-layer GDN tape-replay rollback)")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np  # noqa: F401

    for _ in range(args.warmup):
        cpu_step_sample()
    times = []
    sample = ""
    for _ in range(args.steps):
        t, sample, _ = cpu_step_sample()
        times.append(t)
    t_step = sum(times) / len(times)
    value = 1.0 / t_step
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": workload_name(), "requests_per_gpu": args.requests_per_gpu,
                   "tokens_per_request": 16,
                   "parallelism": "host cores of rank 0 (request-steps/s do not depend on the GPU count)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"dfl_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        out = parse_clock_samples(self.path.read_text())
        self.path.unlink(missing_ok=True)
        return out


def parse_clock_samples(text: str) -> dict:
    """Median SM clock, max SM clock and the throttle reasons seen in the
    sampler's CSV lines (sm, max sm, hw_slowdown, hw_thermal_slowdown,
    sw_thermal_slowdown, sw_power_cap; reasons read "Active" / "Not Active")."""
    sm, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in text.splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 6:
            continue
        try:
            sm.append(float(parts[0]))
            mx = float(parts[1])
        except ValueError:
            continue
        for n, v in zip(names, parts[2:]):
            if v.lower().startswith("active"):
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
            "reasons": sorted(reasons)}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from dflash_mlx_b200.verify_step import VerifyStep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD

    from dflash_mlx_b200.verify_step import StackShape

    shape = StackShape(layers=args.layers)
    step = VerifyStep(dev, requests=args.requests_per_gpu, shape=shape, rank=rank, world=world,
                      group=group, weight_layout=args.weight_layout,
                      fuse_silu=args.weight_layout == "pairs" and not args.no_fuse_silu)
    sh = step.shape
    b = args.requests_per_gpu
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    step.x.copy_(torch.randn(step.x.shape, generator=gen, device=dev).to(torch.bfloat16))
    step.verify_ids.copy_(torch.randint(0, sh.vocab, step.verify_ids.shape, generator=gen, device=dev,
                                        dtype=torch.int64).to(torch.int32))
    step.capture()

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step.run_step()
    barrier()
    evq = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    e0.record(step.stream)
    for i in range(args.steps):
        step.run_step(evq[i])
    e1.record(step.stream)
    barrier()
    clk = clocks.stop()
    t_total = e0.elapsed_time(e1) * 1e-3
    t_qmm = sum(a.elapsed_time(bb) for a, bb in evq) * 1e-3
    # max over ranks
    tt = torch.tensor([t_total, t_qmm], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_total, t_qmm = float(tt[0]), float(tt[1])
    t_step = t_total / args.steps
    value = world * b / t_step

    # end to end through the public API: pinned host inputs in, results out
    x_host = torch.empty(step.x.shape, dtype=torch.bfloat16).pin_memory()
    ids_host = torch.empty(step.verify_ids.shape, dtype=torch.int32).pin_memory()
    x_host.copy_(step.x.cpu())
    ids_host.copy_(step.verify_ids.cpu())
    for _ in range(max(1, args.warmup)):
        step.verify(x_host, ids_host)
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(step.stream)
    out = None
    for _ in range(args.steps):
        out = step.verify(x_host, ids_host)
    f1.record(step.stream)
    barrier()
    te = torch.tensor([f0.elapsed_time(f1) * 1e-3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    t_e2e = float(te[0]) / args.steps
    h2d = x_host.numel() * 2 + ids_host.numel() * 4
    d2h = int(out.numel()) * 4

    # roofline of the dominant kernel (the int4 verify qmm)
    peak, peak_kind = _peaks()
    launches = len(sh.launches()) * sh.layers * (((b + 1) // 2) if step.pack_requests else b)
    bytes_per_step = sh.qmm_bytes_per_step(b, step.pack_requests, silu_fused=step.fuse_silu)
    achieved = bytes_per_step / (t_qmm / args.steps) / 1e9
    traffic, _ = _traffic_per_launch()

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            t_cpu, sample, parts = cpu_step_sample()
            cpu = {"value": 1.0 / t_cpu, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                   "sample": sample}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights with BASELINE distributions; no checkpoints offline)",
            "config": {
                "workload": workload_name(sh.layers),
                "requests_per_gpu": b, "tokens_per_request": sh.block,
                "weight_layout": args.weight_layout,
                "requests_share_launches": step.pack_requests,
                "mlp_silu_fused": step.fuse_silu,
                "parallelism": f"request-DP x{world}, lm_head vocab split x{world}",
                "l2": "inputs larger than L2 (12.3 GB of packed weights per step)",
                "qmm_ms_per_step": t_qmm / args.steps * 1e3,
                "qmm_gbs": achieved,
            },
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "qmm_w4g64 (int4 verify qmm, M=16)",
                         "peak_source": peak_kind,
                         "note": "achieved = algorithmic bytes of the qmm launches of a step (4 per "
                                 "layer: q|k|v, o, gate|up, down) / their CUDA-event time inside "
                                 "the timed region"},
            # ours per step: 4 qmm per layer and request (+ 1 SiLU*up launch unless it
            # is fused into the gate|up epilogue), lm_head argmax, accept, one tape
            # replay over all GDN layers
            "gpu_launches": args.steps * (launches + (0 if step.fuse_silu else launches // 4)
                                          + 2 + 1),
            "e2e": {"value": world * b / t_e2e, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        step.graphs = None
        dist.destroy_process_group()
    return 0


def run_moe(args):
    """BASELINE config 2 on one GPU: the MoE verify layer (hidden 2048, 256
    experts, top-8, expert intermediate 512, one shared expert) at 16 tokens.
    Reports the HBM GB/s of the layer (bytes of the experts the routing
    activates + the shared expert + activations) from CUDA events around a
    graph of ``--moe-layers`` layers with distinct weights (1.9 GB, larger than
    L2).  Not the default workload: the driver's bench line is the verify
    step."""
    import torch

    import __graft_entry__

    __graft_entry__.load_package()
    from dflash_mlx_b200 import moe as M

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"workload": "moe", "unavailable": "the MoE measurement runs on one GPU"}))
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hid, inter, e, topk, tok = 2048, 512, 256, 8, 16
    gen = torch.Generator(device=dev).manual_seed(7)

    def qweight(shape_n, shape_k, lead=()):
        q = torch.randint(-2**31, 2**31 - 1, (*lead, shape_n, shape_k // 8), dtype=torch.int64,
                          generator=gen, device=dev).to(torch.int32)
        sc = torch.rand((*lead, shape_n, shape_k // 64), generator=gen, device=dev) * 0.016 + 0.004
        bi = -8 * sc + torch.randn(sc.shape, generator=gen, device=dev) * 0.1 * sc
        return M.QuantWeight(q, sc.to(torch.bfloat16), bi.to(torch.bfloat16))

    from dflash_mlx_b200.verify_qmm import interleave_gate_up

    layers = []
    for _ in range(args.moe_layers):
        experts = {"gate": qweight(inter, hid, (e,)), "up": qweight(inter, hid, (e,)),
                   "down": qweight(hid, inter, (e,))}
        shared = {"gate": qweight(inter, hid), "up": qweight(inter, hid), "down": qweight(hid, inter)}
        if not args.no_fuse_silu:
            # load-time layout: gate/up interleaved, SiLU*up fused into their launch
            experts = {"gate_up": M.fuse_expert_gate_up(experts["gate"], experts["up"]),
                       "down": experts["down"]}
            g, u = shared["gate"], shared["up"]
            shared = {"gate_up": M.QuantWeight(interleave_gate_up(g.q, u.q).contiguous(),
                                               interleave_gate_up(g.s, u.s).contiguous(),
                                               interleave_gate_up(g.b, u.b).contiguous()),
                      "down": shared["down"]}
        logits = torch.randn((tok, e), generator=gen, device=dev)
        layers.append((experts, shared, logits))
    x = torch.randn((tok, hid), generator=gen, device=dev).to(torch.bfloat16)
    active = []
    for _, _, logits in layers:
        _, _, ids = M.route(logits, topk)
        active.append(int(torch.unique(ids).numel()))
    per_expert = 3 * (inter * hid // 2 + 4 * inter * hid // 64)
    act_bytes = 2 * tok * hid * 2 + 2 * tok * topk * (inter * 2 + hid) + 2 * tok * (3 * inter + hid)
    bytes_total = sum(a * per_expert + per_expert + act_bytes for a in active)
    stream = torch.cuda.Stream(dev)

    def body():
        for experts, shared, logits in layers:
            M.moe_layer(x, logits, experts, shared, top_k=topk)

    with torch.cuda.stream(stream):
        body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / args.steps
    peak, kind = _peaks()
    gbs = bytes_total / t / 1e9
    print(json.dumps({
        "workload": "moe", "metric": "MoE verify layer (BASELINE config 2) HBM GB/s", "value": gbs,
        "unit": "GB/s", "us_per_layer": t / len(layers) * 1e6, "layers": len(layers),
        "active_experts_per_layer": active, "bytes_per_layer": bytes_total / len(layers),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_source": kind},
        "silu_fused": not args.no_fuse_silu, "gpu_launches_per_layer": 6 if not args.no_fuse_silu else 10,
        "steps": args.steps, "warmup": args.warmup, "dtype": "bf16", "data": "synthetic"}))
    return 0


def run_gdn(args):
    """GDN kernels off the bench step, on one GPU, at BASELINE config 4's head
    sizes (48 value heads, Dk = Dv = 128, 16 tokens): the verify forward that
    records the tape (``--workload gdn-forward``, 48 layers in one launch as
    the batch) and the DDTree forward over a 16-node tree
    (``--workload ddtree``, per-node states written).  Reports HBM GB/s of the
    algorithmic bytes (fp32 states in and out, bf16 q/k/v, fp32 g/beta/tape)
    from CUDA events around a CUDA graph of the launch."""
    import numpy as np
    import torch

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"workload": args.workload, "unavailable": "runs on one GPU"}))
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(11)
    hv, hk, dk, dv, t = 48, 16, 128, 128, 16
    b = 48 if args.workload == "gdn-forward" else 4

    def unit(shape):
        a = torch.randn(shape, generator=gen, device=dev)
        return (a / a.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

    q, k = unit((b, t, hk, dk)), unit((b, t, hk, dk))
    v = torch.randn((b, t, hv, dv), generator=gen, device=dev).to(torch.bfloat16)
    g = torch.exp(-torch.nn.functional.softplus(torch.randn((b, t, hv), generator=gen, device=dev)))
    beta = torch.sigmoid(torch.randn((b, t, hv), generator=gen, device=dev))
    state = torch.randn((b, hv, dv, dk), generator=gen, device=dev) * 0.05
    parents = torch.tensor([-1] + [int(x) for x in np.random.default_rng(1).integers(-1, np.arange(1, t))],
                           dtype=torch.int32, device=dev)
    state_bytes = b * hv * dv * dk * 4
    io_bytes = 2 * b * t * hk * dk * 2 + b * t * hv * dv * 2 + 2 * b * t * hv * 4
    if args.workload == "gdn-forward":
        fn = lambda: pkg.gated_delta_kernel_with_tape(q, k, v, g, beta, state)
        alg = 2 * state_bytes + io_bytes + b * t * hv * dv * (2 + 4)       # state in/out, y, tape
        what = "gated_delta_kernel_with_tape, 48 layers x 1 request (layer folded into the batch)"
    else:
        fn = lambda: pkg.gated_delta_tree_kernel(q, k, v, g, beta, state, parents)
        # snapshot read, every node state written and (for non-roots) its parent's read back
        n_reads = int((parents >= 0).sum())
        alg = state_bytes * (1 + t + n_reads) // 1 + io_bytes + b * t * hv * dv * 2
        what = f"gated_delta_tree_kernel, {b} requests x 16-node tree ({n_reads} non-root nodes)"
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / args.steps
    peak, kind = _peaks()
    gbs = alg / sec / 1e9
    print(json.dumps({"workload": args.workload, "metric": f"{what}: HBM GB/s", "value": gbs, "unit": "GB/s",
                      "us_per_launch": sec * 1e6, "bytes_per_launch": alg,
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                   "frac": gbs / peak, "peak_source": kind},
                      "steps": args.steps, "warmup": args.warmup, "data": "synthetic (config 4 distributions)"}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests-per-gpu", type=int, default=1)
    ap.add_argument("--layers", type=int, default=64,
                    help="decoder layers of the qmm stack (64 = the benchmark; fewer only for "
                         "profiling small cases)")
    ap.add_argument("--weight-layout", choices=["mlx", "pairs"], default="pairs",
                    help="int4 nibble order of the stack's weights: the reference's MLX packing, "
                         "or repacked once at load into the kernel's pair-packed order")
    ap.add_argument("--no-fuse-silu", action="store_true",
                    help="run SiLU*up as its own launch after the gate|up projection")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["verify", "moe", "gdn-forward", "ddtree"], default="verify",
                    help="verify: the benchmark's verify step (default); moe: BASELINE config 2; "
                         "gdn-forward / ddtree: the GDN tape producer and the tree kernel alone")
    ap.add_argument("--moe-layers", type=int, default=4)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "moe":
        return run_moe(args)
    if args.workload in ("gdn-forward", "ddtree"):
        return run_gdn(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
