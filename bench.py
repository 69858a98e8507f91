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


def _peak_tflops():
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except Exception:
        return 1590.0


def _profile_value(fname: str, key: str):
    """An integer recorded as ``key value`` in a committed ncu summary."""
    f = ROOT / "profiles" / fname
    try:
        for line in f.read_text().splitlines():
            if line.startswith(key):
                return int(line.split(":")[1].strip()), line
    except Exception:
        pass
    return None, None


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
_CPU_SAMPLE = {}
CPU_ROW_FRACTION = 8   # the CPU sample computes 1/8 of each launch's output rows


def _cpu_sample_inputs():
    """Seeded inputs of the CPU sample, made once per process (input
    generation is not part of the timed sample): 1/8 of the output rows of
    each of the four qmm launch shapes of a decoder layer (q|k|v 8192x5120,
    o 5120x6144, gate|up 34816x5120, down 5120x17408; full K), a 1/64 slice
    of the lm_head vocabulary and one GDN layer's tape."""
    import numpy as np

    from oracle import bf16 as obf16
    from oracle import qmm as oqmm

    if _CPU_SAMPLE:
        return _CPU_SAMPLE
    rng = np.random.default_rng(0)
    layer = []
    for n, k in ((8192, 5120), (5120, 6144), (34816, 5120), (5120, 17408)):
        # 1/CPU_ROW_FRACTION of each launch's output rows, full K
        layer.append((oqmm.synth_x(rng, 16, k), *oqmm.synth_weights(rng, n // CPU_ROW_FRACTION, k)))
    _CPU_SAMPLE["layer"] = layer
    _CPU_SAMPLE["h"] = oqmm.synth_x(rng, 16, 5120)
    _CPU_SAMPLE["lm_w"] = obf16.from_f32((rng.standard_normal((248320 // 64, 5120)) * 0.02)
                                         .astype(np.float32))
    _CPU_SAMPLE["gdn"] = ((rng.standard_normal((1, 48, 128, 128)) * 0.05).astype(np.float32),
                          rng.standard_normal((1, 16, 48, 128)).astype(np.float32),
                          rng.standard_normal((1, 16, 48, 128)).astype(np.float32),
                          rng.random((1, 16, 48)).astype(np.float32))
    _CPU_SAMPLE["rng"] = rng
    return _CPU_SAMPLE


def cpu_step_sample():
    """Time the reference algorithm (oracle restatement, all host threads via
    BLAS) on a bounded sample of one verify step and extrapolate it to the
    full step: 1/8 of the output rows of one decoder layer's four qmm
    launches (x8 x64 layers), the lm_head on 1/64 of the vocabulary (x64) and
    one GDN layer's replay (x48).
    Returns (extrapolated seconds per step, sample text, parts, seconds the
    sample itself took)."""
    import numpy as np

    from oracle import gdn as ogdn
    from oracle import lmhead as olm
    from oracle import qmm as oqmm

    d = _cpu_sample_inputs()
    t0 = time.perf_counter()
    for x, w_q, sc, bi in d["layer"]:
        oqmm.qmm(x, w_q, sc, bi, accum=np.float32)
    t_layer = time.perf_counter() - t0
    t0 = time.perf_counter()
    lg = olm.logits_bf16(d["h"], d["lm_w"])
    post = olm.greedy_tokens(lg).reshape(1, 16)
    ids = olm.synth_verify_ids(d["rng"], post, 248320)
    olm.verify_accept(lg.reshape(1, 16, -1), ids)
    t_lm = time.perf_counter() - t0
    st, kk, tape, g = d["gdn"]
    t0 = time.perf_counter()
    ogdn.tape_replay_accepted(tape, kk, g, st.copy(), np.array([9]))
    t_gdn = time.perf_counter() - t0
    parts = {"qmm_s": t_layer * 64 * CPU_ROW_FRACTION, "lm_head_s": t_lm * 64, "gdn_s": t_gdn * 48}
    total = sum(parts.values())
    sample = ("1/%d of the output rows of each of one decoder layer's four qmm launches (q|k|v, o, "
              "gate|up, down; x%d rows x64 layers), lm_head 16 rows x 3880 vocab (x64), GDN replay "
              "1 layer 48 heads (x48); numpy, %d host threads"
              % (CPU_ROW_FRACTION, CPU_ROW_FRACTION, os.cpu_count()))
    return total, sample, parts, t_layer + t_lm + t_gdn


def workload_name(layers: int = 64) -> str:
    """The verify-step workload both arms time (config.workload)."""
    return (f"verify step = config1 ({layers}-layer int4 g64 qmm stack, hidden 5120, "
            "M=16 per request) + config3 (lm_head 248320x5120 bf16, vocab split over "
            "ranks) + config4 (48-layer GDN tape-replay rollback)")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    for _ in range(args.warmup):
        cpu_step_sample()
    times, sampled = [], []
    sample = ""
    for _ in range(args.steps):
        t, sample, _, t_sample = cpu_step_sample()
        times.append(t)
        sampled.append(t_sample)
    t_step = sum(times) / len(times)
    t_sampled = sum(sampled) / len(sampled)
    value = 1.0 / t_step
    # a step of this arm is the bounded sample (what actually ran, so that
    # steps x ms_per_step is the timed region); value is that sample
    # extrapolated to a whole verify step (extrapolated_ms_per_step)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_sampled * 1e3,
        "extrapolated_ms_per_step": t_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": workload_name(), "requests_per_gpu": args.requests_per_gpu,
                   "tokens_per_request": 16,
                   "parallelism": "host cores of rank 0 (request-steps/s do not depend on the GPU count)",
                   "cpu_baseline_method": "extrapolated from sampled layers",
                   "sampled_s_per_step": t_sampled},
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

    QUERY = ("--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def start(self, first_sample_timeout: float = 10.0):
        """Start sampling every 200 ms; returns once the first sample is in
        (nvidia-smi can take seconds to start when every rank starts one)."""
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), self.QUERY,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t_end = time.time() + first_sample_timeout
        while time.time() < t_end and self.proc.poll() is None:
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.05)

    def _one_shot(self) -> str:
        try:
            return subprocess.run(["nvidia-smi", "-i", str(self.index), self.QUERY,
                                   "--format=csv,noheader,nounits"], capture_output=True,
                                  text=True, timeout=30).stdout
        except Exception:
            return ""

    def stop(self):
        if self.proc is None:
            out = parse_clock_samples(self._one_shot())
            out["sampling"] = "one query after the timed region (sampler did not start)"
            return out
        # one more period so that a short timed region is followed by a sample
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        out = parse_clock_samples(self.path.read_text())
        self.path.unlink(missing_ok=True)
        if out["sm_mhz"] is None:
            out = parse_clock_samples(self._one_shot())
            out["sampling"] = "one query after the timed region (no sample during it)"
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
    from dflash_mlx_b200.verify_step import StackShape, init_process_group

    if world > 1:
        group = init_process_group("nccl", timeout_s=120, device=dev)

    shape = StackShape(layers=args.layers)
    step = VerifyStep(dev, requests=args.requests_per_gpu, shape=shape, rank=rank, world=world,
                      group=group, weight_layout=args.weight_layout,
                      fuse_silu=args.weight_layout != "mlx" and not args.no_fuse_silu,
                      qmm_deps=args.qmm_deps, collectives_in_graph=not args.collectives_eager)
    sh = step.shape
    b = args.requests_per_gpu
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    step.x.copy_(torch.randn(step.x.shape, generator=gen, device=dev).to(torch.bfloat16))
    step.verify_ids.copy_(torch.randint(0, sh.vocab, step.verify_ids.shape, generator=gen, device=dev,
                                        dtype=torch.int64).to(torch.int32))
    step.capture()
    # Config 3's verify ids: the target's true posterior for these hidden rows
    # comes from one step at set-up (same lm_head, same vocabulary split);
    # each draft then equals the previous position's posterior with
    # probability 0.88, else a uniform token, so acceptance lengths (and the
    # rollback's replayed step counts) follow that distribution.
    step.run_step()
    torch.cuda.synchronize(dev)
    step.verify_ids.copy_(synth_verify_ids(step.posterior.clone(), sh.vocab, 0.88, gen))

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

    mean_acc = float(step.acceptance.float().mean())
    # the stack with every projection chained to the one before it, timed
    # outside the loop above (same weights, one plan launch per run)
    t_chain = None
    if step.plan is not None and args.qmm_deps != "chain" and not args.no_extra_configs:
        headline_plan = step.plan
        chained = step._build_plan("chain")
        with torch.cuda.device(dev), torch.cuda.stream(step.stream):
            for _ in range(3):
                chained.run()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(step.stream)
            for _ in range(args.steps):
                chained.run()
            c1.record(step.stream)
        torch.cuda.synchronize(dev)
        t_chain = c0.elapsed_time(c1) / args.steps
        tc = torch.tensor([t_chain], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tc, op=dist.ReduceOp.MAX)
        t_chain = float(tc[0])
        step.plan = headline_plan
        del chained
    # batched requests (every rank, same collectives): 8 requests per GPU, and
    # a fixed global batch of 64 split over the GPUs (strong scaling)
    batched = None
    if step.plan is not None and not args.no_batched:
        batched = measure_batched(step, args, dev, world, rank, group)
    # roofline of the dominant kernel (the int4 verify qmm)
    peak, peak_kind = _peaks()
    plan = step.plan is not None
    per_launch = step.requests_per_launch
    launches = len(sh.launches()) * sh.layers * (-(-b // per_launch))
    bytes_per_step = sh.qmm_bytes_per_step(b, per_launch, silu_fused=step.fuse_silu)
    achieved = bytes_per_step / (t_qmm / args.steps) / 1e9
    qmm_tflops = b * sh.qmm_flops_per_request() / (t_qmm / args.steps) / 1e12
    if plan:
        # one launch runs the whole stack: DRAM bytes of a layer (ncu) x layers
        per_layer, _ = _profile_value("qmm_plan_verify_stack.md", "dram_bytes_per_layer:")
        traffic = None if per_layer is None else per_layer * sh.layers
        qmm_launches = 1
    else:
        traffic, _ = _traffic_per_launch()
        qmm_launches = launches + (0 if step.fuse_silu else launches // 4)

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            t_cpu, sample, parts, _ = cpu_step_sample()
            cpu = {"value": 1.0 / t_cpu, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                   "sample": sample, "method": "extrapolated from sampled layers"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights with BASELINE distributions; no checkpoints offline)",
            "config": {
                "workload": workload_name(sh.layers),
                "requests_per_gpu": b, "tokens_per_request": sh.block,
                "weight_layout": args.weight_layout,
                "requests_per_weight_read": per_launch,
                "qmm_launch": (("one plan launch per step; each projection waits on the device "
                                "for the projections whose outputs it reads (down for gate|up's "
                                "SiLU output, the next layer's q|k|v for this layer's down); o "
                                "and gate|up read stand-ins for the attention output and the "
                                "normalised residual (ops outside this path)")
                               if plan and args.qmm_deps == "dataflow" else
                               "one plan launch per step; every projection waits for the one "
                               "before it" if plan else
                               "one launch per projection (programmatic dependent launch)"),
                "qmm_ms_per_step_chained": t_chain,
                "mlp_silu_fused": step.fuse_silu,
                "parallelism": f"request-DP x{world}, lm_head vocab split x{world}",
                "collectives": ("all-gathers captured in the step's second CUDA graph"
                                if world > 1 and step.collectives_in_graph else
                                "host-issued between CUDA graphs" if world > 1 else "none"),
                "l2": "inputs larger than L2 (12.4 GB of packed weights per step)",
                "qmm_ms_per_step": t_qmm / args.steps * 1e3,
                "qmm_gbs": achieved,
                "qmm_tflops": qmm_tflops,
                "qmm_tensor_frac": qmm_tflops / _peak_tflops(),
                "verify_ids": "P(draft = previous position's posterior) = 0.88, posterior from set-up",
                "mean_acceptance": mean_acc,
            },
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": ("qmm_plan_kernel (int4 verify qmm, M=16: the step's %d "
                                    "projections in one persistent launch)" % (4 * sh.layers)
                                    if plan else "qmm_w4g64 (int4 verify qmm, M=16)"),
                         "peak_source": peak_kind,
                         "note": "achieved = algorithmic bytes of the step's projections (4 per "
                                 "layer: q|k|v, o, gate|up + SiLU, down; packed weights + bf16 "
                                 "scales/biases + activations) / their CUDA-event time inside "
                                 "the timed region; traffic = ncu DRAM bytes per launch"},
            # ours per step: the qmm stack (one plan launch, or 4 launches per layer
            # and request pair, + 1 SiLU*up launch unless fused), lm_head argmax,
            # accept, one tape replay over all GDN layers
            "gpu_launches": args.steps * (qmm_launches + 2 + 1),
            "e2e": {"value": world * b / t_e2e, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if batched is not None:
            line["config"].update(batched)
        if world == 1 and not args.no_extra_configs:
            # the other configurations, measured in this process after the
            # timed loop (each in its own CUDA graph, CUDA events)
            del step
            torch.cuda.empty_cache()
            line["config"].update(measure_other_configs(dev, args))
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        step.graphs = None
        dist.destroy_process_group()
    return 0


def measure_batched(step, args, dev, world: int, rank: int, group) -> dict:
    """Verify steps with several requests per GPU, on every rank (the same
    collectives in the same order), reusing ``step``'s weights:

    * ``batched_b8``: 8 requests per GPU (one 128-row token tile: the 8
      requests share one read of every weight), whole-job requests/s;
    * ``strong_b64``: a fixed global batch of 64 requests split over the
      GPUs (64 / N per GPU), requests/s -- v_N / (N v_1) is the strong-scaling
      efficiency.

    Each: its own CUDA graphs, P = 0.88 verify ids from its own posterior,
    3 warm-up steps, then min(steps, 5) steps between CUDA events; the step
    time and the qmm stack's time are maxima over ranks."""
    import torch
    import torch.distributed as dist

    from dflash_mlx_b200.verify_step import VerifyStep

    sh = step.shape
    cases = [("batched_b8", 8)]
    if args.strong_batch % world == 0:
        cases.append((f"strong_b{args.strong_batch}", args.strong_batch // world))
    steps = max(1, min(args.steps, 5))
    tflops = _peak_tflops()
    peak, _ = _peaks()
    out = {}
    for name, b in cases:
        s2 = VerifyStep(dev, requests=b, shape=sh, rank=rank, world=world, group=group,
                        weight_layout=step.weight_layout, fuse_silu=step.fuse_silu,
                        qmm_deps=step.qmm_deps, share_weights=step,
                        collectives_in_graph=step.collectives_in_graph)
        gen = torch.Generator(device=dev).manual_seed(300 + rank)
        s2.x.copy_(torch.randn(s2.x.shape, generator=gen, device=dev).to(torch.bfloat16))
        s2.verify_ids.copy_(torch.randint(0, sh.vocab, s2.verify_ids.shape, generator=gen, device=dev,
                                          dtype=torch.int64).to(torch.int32))
        s2.capture()
        s2.run_step()
        torch.cuda.synchronize(dev)
        s2.verify_ids.copy_(synth_verify_ids(s2.posterior.clone(), sh.vocab, 0.88, gen))
        for _ in range(3):
            s2.run_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        evq = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s2.stream)
        for i in range(steps):
            s2.run_step(evq[i])
        e1.record(s2.stream)
        torch.cuda.synchronize(dev)
        tt = torch.tensor([e0.elapsed_time(e1) * 1e-3, sum(a.elapsed_time(c) for a, c in evq) * 1e-3],
                          dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_step, t_qmm = float(tt[0]) / steps, float(tt[1]) / steps
        by = sh.qmm_bytes_per_step(b, s2.requests_per_launch, silu_fused=s2.fuse_silu)
        fl = b * sh.qmm_flops_per_request()
        out[name] = {"requests_per_gpu": b, "global_requests": b * world,
                     "requests_per_s": world * b / t_step, "ms_per_step": t_step * 1e3,
                     "qmm_ms_per_step": t_qmm * 1e3, "qmm_tflops": fl / t_qmm / 1e12,
                     "qmm_tensor_frac": fl / t_qmm / 1e12 / tflops, "qmm_hbm_frac": by / t_qmm / 1e9 / peak,
                     "mean_acceptance": float(s2.acceptance.float().mean()), "steps": steps}
        s2.graphs = None
        del s2
        torch.cuda.empty_cache()
    out["batched_note"] = ("measured after the timed loop on every rank; requests_per_s is whole-job "
                           "(all GPUs); fractions of the measured cuBLAS bf16 burst / HBM copy peaks")
    return out


def synth_verify_ids(posterior, vocab: int, p_match: float, gen):
    """verify_ids [B, T] for posterior [B, T]: position 0 uniform, position j
    the posterior of position j - 1 with probability p_match, else uniform."""
    import torch

    b, t = posterior.shape
    dev = posterior.device
    ids = torch.randint(0, vocab, (b, t), generator=gen, device=dev, dtype=torch.int64).to(torch.int32)
    hit = torch.rand((b, t), generator=gen, device=dev) < p_match
    ids[:, 1:] = torch.where(hit[:, 1:], posterior[:, :-1].to(torch.int32), ids[:, 1:])
    return ids


def _graph_time(fn, dev, reps: int, warmup: int = 3) -> float:
    """Seconds per call of ``fn`` captured once in a CUDA graph and replayed
    ``reps`` times between CUDA events on the capturing stream."""
    import torch

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        for _ in range(warmup):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    del graph
    return e0.elapsed_time(e1) / 1e3 / reps


def measure_other_configs(dev, args) -> dict:
    """BASELINE configs 0, 2, 4 and config 3 at B = 16 / 128 on one GPU, each
    with its roofline fraction (of the measured peaks):

    * config0: 16 x 4096 x 4096 int4 verify qmm (MLX packing, the drop-in
      entry), 64 calls over 64 distinct weight copies (621 MB > L2) per graph;
      config0_plan: the same 64 products as one 64-phase projection plan;
    * moe: the config-2 MoE layer (4 layers with distinct weights per graph);
    * rollback_config4: tape replay of 64 sequences x 48 layers (a ~ U{0..16}
      per sequence, Hk = Hv = 48), in place, one launch;
    * lmhead_b16 / lmhead_b128: argmax keys of 256 / 2048 hidden rows over the
      full 248,320 x 5120 vocabulary (tensor-bound at B = 128)."""
    import torch

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from dflash_mlx_b200.verify_qmm import qmm_w4g64

    peak, _ = _peaks()
    tflops = _peak_tflops()
    out = {}
    gen = torch.Generator(device=dev).manual_seed(17)
    # config 0
    m, k, n, copies = 16, 4096, 4096, 64
    ws = []
    for _ in range(copies):
        q = torch.randint(-2**31, 2**31 - 1, (n, k // 8), dtype=torch.int64, generator=gen,
                          device=dev).to(torch.int32)
        sc = torch.rand((n, k // 64), generator=gen, device=dev) * 0.016 + 0.004
        bi = -8 * sc + torch.randn(sc.shape, generator=gen, device=dev) * 0.1 * sc
        ws.append((q, sc.to(torch.bfloat16), bi.to(torch.bfloat16)))
    x0 = torch.randn((m, k), generator=gen, device=dev).to(torch.bfloat16)
    y0 = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

    def cfg0():
        for q, sc, bi in ws:
            qmm_w4g64(x0, q, sc, bi, out=y0)

    t = _graph_time(cfg0, dev, reps=10) / copies
    b0 = n * k // 2 + 4 * n * (k // 64) + 2 * m * (k + n)
    out["config0_qmm_us"] = t * 1e6
    out["config0_qmm_gbs"] = b0 / t / 1e9
    out["config0_qmm_frac"] = b0 / t / 1e9 / peak
    # the same 64 calls as one projection plan (tiled copies of the weights,
    # 64 independent phases in one launch)
    from dflash_mlx_b200 import qmm_plan as QP
    tiled = [QP.tile_weight(q, sc, bi) for q, sc, bi in ws]
    del ws
    ys = [torch.empty((m, n), dtype=torch.bfloat16, device=dev) for _ in tiled]
    plan0 = QP.ProjectionPlan([QP.PlanPhase(x0, w, yy) for w, yy in zip(tiled, ys)])
    t = _graph_time(plan0.run, dev, reps=10) / copies
    out["config0_plan_us"] = t * 1e6
    out["config0_plan_gbs"] = b0 / t / 1e9
    out["config0_plan_frac"] = b0 / t / 1e9 / peak
    del tiled, plan0, ys
    # config 2
    moe = measure_moe(dev, layers=4, steps=10, warmup=3, fuse_silu=True)
    out["moe_layer_us"] = moe["us_per_layer"]
    out["moe_layer_gbs"] = moe["value"]
    out["moe_layer_frac"] = moe["roofline"]["frac"]
    # config 4 at 64 sequences x 48 layers
    seqs, layers, hv, dk, dv, tt = 64, 48, 48, 128, 128, 16
    lb = seqs * layers
    state = torch.randn((lb, hv, dv, dk), generator=gen, device=dev) * 0.05
    tape = torch.randn((lb, tt, hv, dv), generator=gen, device=dev)
    kk = torch.randn((lb, tt, hv, dk), generator=gen, device=dev)
    kk = (kk / kk.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    g = torch.exp(-torch.nn.functional.softplus(torch.randn((lb, tt, hv), generator=gen, device=dev)))
    a = torch.randint(0, tt + 1, (seqs,), generator=gen, device=dev, dtype=torch.int32)
    steps = a.repeat(layers)
    t = _graph_time(lambda: pkg.tape_replay_(state, tape, kk, g, steps), dev, reps=5)
    a_host = a.cpu().long()
    per_step = hv * dv * 4 + hv * dk * 2 + hv * 4
    b4 = layers * int(((a_host > 0).long() * 2 * hv * dv * dk * 4 + a_host * per_step).sum())
    out["rollback_config4_us"] = t * 1e6
    out["rollback_config4_gbs"] = b4 / t / 1e9
    out["rollback_config4_frac"] = b4 / t / 1e9 / peak
    del state, tape, kk, g
    # config 3 at B = 16 and 128 on the full vocabulary (one GPU)
    v, d = 248320, 5120
    w = (torch.randn((v, d), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    for bsz in (16, 128):
        h = torch.randn((bsz * 16, d), generator=gen, device=dev).to(torch.bfloat16)
        keys = torch.empty(bsz * 16, dtype=torch.int64, device=dev)
        t = _graph_time(lambda: pkg.lm_head_argmax_keys(h, w, out=keys), dev, reps=5)
        fl = 2.0 * bsz * 16 * v * d
        by = v * d * 2 + bsz * 16 * d * 2
        out[f"lmhead_b{bsz}_ms"] = t * 1e3
        out[f"lmhead_b{bsz}_hbm_frac"] = by / t / 1e9 / peak
        out[f"lmhead_b{bsz}_tensor_frac"] = fl / t / 1e12 / tflops
    out["other_configs_note"] = ("measured after the timed loop, one CUDA graph each; fractions of "
                                 "the measured HBM copy bandwidth / cuBLAS bf16 burst throughput")
    return out


def measure_moe(dev, layers: int, steps: int, warmup: int, fuse_silu: bool, plan: bool = True) -> dict:
    """BASELINE config 2 (hidden 2048, 256 experts, top-8, intermediate 512,
    one shared expert, 16 tokens): ``layers`` layers with distinct weights in
    one CUDA graph; HBM GB/s of the bytes of the experts the routing
    activates + the shared expert + activations.  ``plan``: each layer's
    expert projections in one plan launch (MoEPlanLayer: route, sort, plan,
    combine); otherwise the per-launch path (moe_layer)."""
    import torch

    import __graft_entry__

    __graft_entry__.load_package()
    from dflash_mlx_b200 import moe as M
    from dflash_mlx_b200.verify_qmm import interleave_gate_up

    hid, inter, e, topk, tok = 2048, 512, 256, 8, 16
    gen = torch.Generator(device=dev).manual_seed(7)

    def qweight(shape_n, shape_k, lead=()):
        q = torch.randint(-2**31, 2**31 - 1, (*lead, shape_n, shape_k // 8), dtype=torch.int64,
                          generator=gen, device=dev).to(torch.int32)
        sc = torch.rand((*lead, shape_n, shape_k // 64), generator=gen, device=dev) * 0.016 + 0.004
        bi = -8 * sc + torch.randn(sc.shape, generator=gen, device=dev) * 0.1 * sc
        return M.QuantWeight(q, sc.to(torch.bfloat16), bi.to(torch.bfloat16))

    lay = []
    for _ in range(layers):
        experts = {"gate": qweight(inter, hid, (e,)), "up": qweight(inter, hid, (e,)),
                   "down": qweight(hid, inter, (e,))}
        shared = {"gate": qweight(inter, hid), "up": qweight(inter, hid), "down": qweight(hid, inter)}
        if fuse_silu:
            # load-time layout: gate/up interleaved, SiLU*up fused into their launch
            experts = {"gate_up": M.fuse_expert_gate_up(experts["gate"], experts["up"]),
                       "down": experts["down"]}
            g, u = shared["gate"], shared["up"]
            shared = {"gate_up": M.QuantWeight(interleave_gate_up(g.q, u.q).contiguous(),
                                               interleave_gate_up(g.s, u.s).contiguous(),
                                               interleave_gate_up(g.b, u.b).contiguous()),
                      "down": shared["down"]}
        logits = torch.randn((tok, e), generator=gen, device=dev)
        lay.append((experts, shared, logits))
    x = torch.randn((tok, hid), generator=gen, device=dev).to(torch.bfloat16)
    active = []
    for _, _, logits in lay:
        _, _, ids = M.route(logits, topk)
        active.append(int(torch.unique(ids).numel()))
    per_expert = 3 * (inter * hid // 2 + 4 * inter * hid // 64)
    act_bytes = 2 * tok * hid * 2 + 2 * tok * topk * (inter * 2 + hid) + 2 * tok * (3 * inter + hid)
    bytes_total = sum(a * per_expert + per_expert + act_bytes for a in active)

    if plan:
        runners = [(M.MoEPlanLayer(experts, shared, tokens=tok, top_k=topk), logits)
                   for experts, shared, logits in lay]

        def body():
            for layer, logits in runners:
                layer(x, logits)
    else:
        def body():
            for experts, shared, logits in lay:
                M.moe_layer(x, logits, experts, shared, top_k=topk)

    t = _graph_time(body, dev, reps=steps, warmup=warmup)
    peak, kind = _peaks()
    gbs = bytes_total / t / 1e9
    return {
        "workload": "moe", "metric": "MoE verify layer (BASELINE config 2) HBM GB/s", "value": gbs,
        "unit": "GB/s", "us_per_layer": t / layers * 1e6, "layers": layers,
        "active_experts_per_layer": active, "bytes_per_layer": bytes_total / layers,
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                     "peak_source": kind},
        "silu_fused": fuse_silu or plan, "path": "plan" if plan else "per-launch",
        "gpu_launches_per_layer": 4 if plan else (6 if fuse_silu else 10),
        "steps": steps, "warmup": warmup, "dtype": "bf16", "data": "synthetic"}


def run_moe(args):
    """BASELINE config 2 on one GPU (see measure_moe).  Not the default
    workload: the driver's bench line is the verify step, which also carries
    this measurement in its config."""
    import torch

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"workload": "moe", "unavailable": "the MoE measurement runs on one GPU"}))
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    print(json.dumps(measure_moe(dev, args.moe_layers, args.steps, args.warmup,
                                 fuse_silu=not args.no_fuse_silu, plan=not args.moe_per_launch)))
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
    ap.add_argument("--weight-layout", choices=["mlx", "pairs", "tiled"], default="tiled",
                    help="int4 layout of the stack's weights: the reference's MLX packing or the "
                         "pair-packed order (one qmm launch per projection), or the tiled layout "
                         "(the whole stack as one projection plan: one persistent launch per step)")
    ap.add_argument("--qmm-deps", choices=["dataflow", "chain"], default="dataflow",
                    help="tiled layout: dataflow = each projection waits only for the projections "
                         "whose outputs it reads; chain = every projection also waits for the one "
                         "before it")
    ap.add_argument("--no-fuse-silu", action="store_true",
                    help="run SiLU*up as its own launch after the gate|up projection")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--collectives-eager", action="store_true",
                    help="N > 1: issue the lm_head all-gathers from the host between CUDA graphs "
                         "instead of capturing them in the step graph")
    ap.add_argument("--no-batched", action="store_true",
                    help="skip the batched-request measurements (8 per GPU, and a fixed global "
                         "batch split over the GPUs) carried in the line's config")
    ap.add_argument("--strong-batch", type=int, default=64,
                    help="global batch of the strong-scaling measurement (split over the GPUs)")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="skip the config 0 / 2 / 4 and lm_head B=16/128 measurements that the "
                         "one-GPU line carries in its config")
    ap.add_argument("--workload", choices=["verify", "moe", "gdn-forward", "ddtree"], default="verify",
                    help="verify: the benchmark's verify step (default); moe: BASELINE config 2; "
                         "gdn-forward / ddtree: the GDN tape producer and the tree kernel alone")
    ap.add_argument("--moe-layers", type=int, default=4)
    ap.add_argument("--moe-per-launch", action="store_true",
                    help="moe workload: one launch per projection instead of one plan per layer")
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
