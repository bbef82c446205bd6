"""Benchmark of siliconfer's Q4Linear path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 7b|70b|0.5b] [--batch T]

Workload (default, N=1): BASELINE config 3 -- a 7B-shaped decode step, 32
layers x 7 projections (hidden 4096, intermediate 11008), symmetric int4,
group 128, seeded N(0, 0.02) weights quantized on the device with the
reference's RTN (bit-exact with pack_weights_sym), fp16 activations N(0,1),
fp32 outputs.  One step = all 224 GEMVs, replayed as one CUDA graph.  The
weights (3.44 GB) are far larger than L2 (126 MB), so every step streams them
from HBM; no flush is needed.

metric/value: algorithmic bytes per step / device time per step, in GB/s
(the reference's formula, scripts/benchmark.py:97-102, extended with the
output).  decode_step_us is the same step as latency.

With N > 1 (torchrun) every rank runs the same workload on its own GPU
(replicas, weak scaling).  --workload 70b selects BASELINE config 5 instead:
the 70B-shaped step sharded over the N GPUs (column-parallel q/k/v/gate/up,
row-parallel o/down with an all-reduce after each; strong scaling), timed with
this library's NVLink peer all-reduce and with NCCL.

--impl reference times the reference's own CPU kernels (oracle/_ref, built
from the reference sources; else the oracle's C port) on the host cores with
every thread, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

HIDDEN = {"7b": (4096, 11008, 32), "70b": (8192, 28672, 80), "0.5b": (896, 4864, 24)}
KV_OUT = {"7b": 4096, "70b": 1024, "0.5b": 128}
PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def shapes(workload: str):
    """(name, N, K) of one layer's projections."""
    h, f, _ = HIDDEN[workload]
    kv = KV_OUT[workload]
    return [("q", h, h), ("k", kv, h), ("v", kv, h), ("o", h, h),
            ("gate", f, h), ("up", f, h), ("down", h, f)]


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        mhz, maxm, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                mhz.append(float(parts[1]))
                maxm = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        out = {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": maxm,
               "reasons": sorted(reasons), "samples": len(mhz)}
        if not mhz:
            out["sampler_output"] = " | ".join(self.lines[:3])[:300]
        return out


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def build_layers(workload, device, tp_rank=0, tp_size=1, seed=1234, n_layers=0):
    """Random-init projections of the named architecture, quantized on the GPU."""
    import torch
    from siliconfer_b200.q4_linear import Q4Linear
    from siliconfer_b200.quant import pack_weights_device
    n_layers = n_layers or HIDDEN[workload][2]
    layers = []
    gen = torch.Generator(device=device)
    for li in range(n_layers):
        for pi, (name, n, k) in enumerate(shapes(workload)):
            gen.manual_seed(seed + 1000 * li + pi)
            row_parallel = name in ("o", "down")
            if tp_size > 1:
                if row_parallel:
                    k = k // tp_size
                else:
                    n = n // tp_size
            W = torch.randn((n, k), generator=gen, device=device) * 0.02
            p, s = pack_weights_device(W, 128)
            del W
            layers.append(Q4Linear(p, s, group_size=128, device=device))
    torch.cuda.synchronize(device)
    return layers


def workload_config(args, world, n_layers, layout):
    """The `config` object of both arms' lines (the same workload)."""
    return {"workload": f"BASELINE config 3: {args.workload}-shaped decode step, "
                        f"{n_layers} layers x 7 projections, each reading its own pre-supplied input",
            "batch": args.batch, "group_size": 128, "layout": layout,
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "weights 3.44 GB per step >> 126 MB L2 (no flush needed)"
            if args.workload == "7b" else "weights >> L2 (no flush needed)",
            "layer_order": "decode_step_us_layer_order: same step with q/k/v -> o -> "
                           "gate/up -> down -> next layer dependencies inside the launch"}


def run_ours(args, rank, world, local_rank):
    import torch
    from siliconfer_b200 import _lib
    from siliconfer_b200.runner import Q4StepRunner

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)

    t_build = time.perf_counter()
    layers = build_layers(args.workload, device, n_layers=args.layers)
    # Headline workload (the measurement table's config 3): every projection
    # reads its own pre-supplied activation -- attention, norms and SwiGLU
    # between projections are outside the Q4Linear path.
    runner = Q4StepRunner(layers, tokens=args.batch, x_dtype=torch.float16,
                          y_dtype=torch.float32, pdl=True, device=device,
                          waits=[False] * len(layers))
    g = torch.Generator(device=device)
    g.manual_seed(7)
    runner.x.copy_(torch.randn(runner.x.shape, generator=g, device=device).to(runner.x.dtype))
    runner.x_host.copy_(runner.x.cpu())
    runner.capture()
    # The same projections in the decoder's order: q/k/v, then o, then
    # gate/up, then down, then the next layer, each phase reading its input
    # only after the previous phase has written its outputs.
    ordered = Q4StepRunner(layers, tokens=args.batch, x_dtype=torch.float16,
                           y_dtype=torch.float32, pdl=True, device=device)
    ordered.x.copy_(runner.x)
    ordered.capture()
    build_s = time.perf_counter() - t_build

    def barrier():
        if dist is not None:
            dist.barrier()

    def timed(replay, n):
        """Device time per replay (ms), CUDA events on the runner's stream."""
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(runner.stream)
        for _ in range(n):
            replay()
        s1.record(runner.stream)
        s1.synchronize()
        return s0.elapsed_time(s1) / n

    # ---- device-resident timing -------------------------------------------
    for _ in range(args.warmup):
        runner.run()
    runner.stream.synchronize()
    barrier()
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    with ClockSampler(local_rank) as clocks:
        # keep the GPU under the same load until the sampler is producing
        t_end = time.perf_counter() + 5.0
        while len(clocks.lines) < 2 and time.perf_counter() < t_end:
            for _ in range(20):
                runner.run()
            runner.stream.synchronize()
        n_before = len(clocks.lines)
        start.record(runner.stream)
        for _ in range(args.steps):
            runner.run()
        stop.record(runner.stream)
        stop.synchronize()
        t_end = time.perf_counter() + 2.0
        while len(clocks.lines) <= n_before and time.perf_counter() < t_end:
            for _ in range(20):
                runner.run()
            runner.stream.synchronize()
    barrier()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(stop) / args.steps
    host_launches = _lib.launch_count() - launches0   # 0: graph replays launch on the device

    # the GEMV kernel alone (roofline), and the decoder-ordered step
    with torch.cuda.stream(runner.stream):
        kernel_ms = timed(runner.graph.replay, args.steps)   # the step is one launch of the GEMV kernel
        for _ in range(args.warmup):
            ordered.graph.replay()
        ordered_ms = timed(ordered.graph.replay, args.steps)
    runner.run()                       # leave the workspace in a full-run state
    runner.stream.synchronize()
    dev_err = _lib.load().sf_q4_check_device_error()
    if dev_err != 0:
        raise RuntimeError(f"device-side wait expired during the bench (status {dev_err})")

    # ---- end to end: pinned host in, pinned host out -------------------------
    for _ in range(max(1, args.warmup)):
        runner.run_host()
    runner.stream.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(runner.stream)
    for _ in range(args.steps):
        runner.run_host()
    e1.record(runner.stream)
    e1.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    if dist is not None:
        t = torch.tensor([ms, e2e_ms, kernel_ms, ordered_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, kernel_ms, ordered_ms = t.tolist()

    step_bytes = runner.algorithmic_bytes()
    total_bytes = step_bytes * world
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    kernel_gbs = step_bytes / (kernel_ms * 1e-3) / 1e9
    xin = runner.x.numel() * runner.x.element_size()
    yout = runner.y.numel() * runner.y.element_size()
    layout = "asym" if layers[0].is_asym else "sym"

    result = {
        "metric": f"int4 GEMV HBM GB/s, {args.workload} decode step (batch {args.batch})",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "decode_step_us": round(ms * 1e3, 2),
        "decode_step_us_layer_order": round(ordered_ms * 1e3, 2),
        "value_layer_order": round(step_bytes * world / (ordered_ms * 1e-3) / 1e9, 1),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4 weights (u8 nibbles) x fp16 activations, exact int32 products, fp32 accumulate",
        "data": "synthetic: seeded N(0,0.02) weights, RTN int4 sym g128 (device pack, bit-exact "
                "with the reference packer); fp16 N(0,1) activations",
        "config": workload_config(args, world, len(layers) // 7, layout),
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(kernel_gbs / peak, 4),
                     "peak_kind": peak_kind,
                     "kernel": f"q4_tile_kernel<{args.batch},{layout},16> (one launch per step)",
                     "bytes_per_launch": step_bytes,
                     "launch_us": round(kernel_ms * 1e3, 2),
                     "traffic": traffic_from_profile(args.workload, args.batch)},
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms, 5),
                "h2d_bytes_per_step": xin, "d2h_bytes_per_step": yout,
                "api": "siliconfer_b200.runner.Q4StepRunner.run_host (pinned host in/out)"},
        "gpu_launches": runner.kernels_per_step * args.steps,
        "host_launch_calls_in_timed_region": host_launches,
        "clocks": clocks.summary(),
        "build_s": round(build_s, 1),
    }
    if world == 1 and args.workload == "7b" and not args.no_prefill:
        result["sweep"] = sweep_measure(layers, device, args)
        result["small_configs"] = small_configs_measure(device)
        result["int2"] = int2_measure(device, args)
        result["per_call"] = per_call_measure(device)
        result["prefill"] = prefill_measure(device, runner.stream)
        result["kv_attention"] = kv_attention_measure(device, runner.stream)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args, layers)
    cleanup = None
    if args.workload == "7b" and not args.no_tp70b:
        # BASELINE config 5 beside the headline: the 70B step sharded over these
        # N GPUs (strong scaling), with its parity check
        del runner, ordered, layers
        torch.cuda.empty_cache()
        result["tp70b"], cleanup = tp_measure(args, rank, world, local_rank, dist)
    if rank == 0:
        print(json.dumps(result), flush=True)
    _exit_watchdog()
    if cleanup is not None:
        cleanup()
    if dist is not None:
        dist.destroy_process_group()


TP_BLOCKS = 8   # weights are drawn in 8 blocks along the sharded dimension: the same matrix at any TP 1/2/4/8


def _tp_weight(workload, li, pi, device, blocks, seed=1234):
    """Rank's shard of projection (li, pi), fp32 on `device`: the concatenation
    of `blocks` (out of TP_BLOCKS) -- row blocks for column-parallel
    projections, whole-group column blocks for row-parallel ones.  Every block
    has its own seed, so the unsharded matrix is the same for every world size."""
    import torch
    name, n, k = shapes(workload)[pi]
    row_parallel = name in ("o", "down")
    gen = torch.Generator(device=device)
    parts = []
    for b in blocks:
        gen.manual_seed(seed + 16 * (7 * li + pi) + b)
        shape = (n, k // TP_BLOCKS) if row_parallel else (n // TP_BLOCKS, k)
        parts.append(torch.randn(shape, generator=gen, device=device) * 0.02)
    return torch.cat(parts, dim=1 if row_parallel else 0), row_parallel


def _tp_x(li, pi, k_full, tokens, device):
    """Unsharded input of projection (li, pi): the same on every rank."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(900_000 + 7 * li + pi + 7919 * tokens)
    return torch.randn((tokens, k_full), generator=gen, device=device).to(torch.bfloat16)


def _dequant_ref(packed, scales, gs):
    """fp32 dequant of a symmetric packed triple in torch (w = q * s, the
    reference's dequantize_sym arithmetic: one exact product per weight)."""
    import torch
    n = packed.shape[0]
    lo = (packed & 15).to(torch.int16)
    hi = (packed >> 4).to(torch.int16)
    q = torch.stack([lo, hi], dim=-1).reshape(n, -1)
    q = torch.where(q >= 8, q - 16, q).float()
    return (q.reshape(n, -1, gs) * scales[:, :, None]).reshape(n, -1)


def tp_measure(args, rank, world, local_rank, dist):
    """the 70B-shaped decode step sharded over `world` GPUs.

    q/k/v/gate/up column-parallel, o/down row-parallel with one all-reduce of
    [batch, 8192] after each (160 per step).  Times, as device time and max
    over ranks:
      fused          the whole step as ONE persistent launch per GPU, every
                     projection reading its own pre-supplied input, the
                     all-reduces fused in (tiles pushed over NVLink);
      fused_ordered  the same launch with the decoder's dependencies: q/k/v ->
                     o -> o all-reduce -> gate/up -> down -> down all-reduce ->
                     next layer, each phase waiting for the one before;
      peer / nccl    one launch per half layer + this library's peer
                     all-reduce kernel, or + NCCL (world > 1);
      fused_batch8   the independent fused step at batch 8.
    Parity: the all-reduced o and down outputs of the first and last layers
    (every row) against an fp64 product of the unsharded weights' fp32
    dequant, for the fused, ordered and NCCL runs; tolerance 1e-3 normwise."""
    import torch
    from siliconfer_b200 import _lib
    from siliconfer_b200.q4_linear import Q4Linear
    from siliconfer_b200.quant import pack_weights_device
    from siliconfer_b200.tensor_parallel import PeerComm, TPStepRunner

    workload = "70b"
    device = torch.device("cuda", local_rank)
    if TP_BLOCKS % world:
        return ({"unavailable": f"the 70B weights are drawn in {TP_BLOCKS} blocks; world {world} does not "
                                f"divide them"}, lambda: None)
    n_layers = args.tp_layers or HIDDEN[workload][2]
    hidden = HIDDEN[workload][0]
    blocks = range(rank * TP_BLOCKS // world, (rank + 1) * TP_BLOCKS // world)
    t_build = time.perf_counter()
    groups = []
    for li in range(n_layers):
        lay = []
        for pi in range(7):
            W, _ = _tp_weight(workload, li, pi, device, blocks)
            p, s_ = pack_weights_device(W, 128)
            del W
            lay.append(Q4Linear(p, s_, group_size=128, device=device))
        groups.append(lay)
    torch.cuda.synchronize(device)
    comm = None
    if world > 1:
        arena = 2 * TPStepRunner.arena_bytes(n_layers, 1, hidden, world) + \
            TPStepRunner.arena_bytes(n_layers, 8, hidden, world)
        comm = PeerComm(slot_bytes=max(1 << 20, 8 * hidden * 4), arena_bytes=arena)
    runners = {
        "fused": TPStepRunner(groups, tokens=1, x_dtype=torch.bfloat16, mode="fused", comm=comm, device=device),
        "fused_ordered": TPStepRunner(groups, tokens=1, x_dtype=torch.bfloat16, mode="fused", comm=comm,
                                      device=device, ordered=True),
        "fused_batch8": TPStepRunner(groups, tokens=8, x_dtype=torch.bfloat16, mode="fused", comm=comm,
                                     device=device),
    }
    if world > 1:
        # the same fused launch without the exchange (partials kept local): what the GEMVs alone cost
        runners["fused_no_exchange"] = TPStepRunner(groups, tokens=1, x_dtype=torch.bfloat16, mode="fused",
                                                    device=device, exchange=False)
        runners["peer"] = TPStepRunner(groups, tokens=1, x_dtype=torch.bfloat16, mode="peer", comm=comm,
                                       device=device)
        runners["nccl"] = TPStepRunner(groups, tokens=1, x_dtype=torch.bfloat16, mode="nccl", device=device)
    # inputs: the unsharded x of every projection, sliced to this rank's K block where row-parallel
    for r in runners.values():
        for li in range(n_layers):
            for pi in range(7):
                name, n, k = shapes(workload)[pi]
                xf = _tp_x(li, pi, k, r.tokens, device)
                if name in ("o", "down"):
                    k0 = rank * k // world
                    xf = xf[:, k0:k0 + k // world]
                xo = r.slots[li][pi][0]
                r.x[xo:xo + xf.numel()].copy_(xf.reshape(-1))
        r.x_host.copy_(r.x.cpu())
    if dist is not None:
        torch.cuda.synchronize(device)
        dist.barrier()   # every rank has built its shards before any exchange kernel runs
    for r in runners.values():
        r.capture()
    build_s = time.perf_counter() - t_build

    def barrier():
        if dist is not None:
            dist.barrier()
            torch.cuda.synchronize(device)

    def timed(r, n):
        for _ in range(args.warmup):
            r.run()
        r.stream.synchronize()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(r.stream)
        for _ in range(n):
            r.run()
        s1.record(r.stream)
        s1.synchronize()
        barrier()
        return s0.elapsed_time(s1) / n

    steps = max(5, min(args.steps, 20))
    times = {name: timed(r, steps) for name, r in runners.items()}
    # end to end through the fused step: pinned host activations in, all-reduced outputs out
    main_r = runners["fused"]
    for _ in range(args.warmup):
        main_r.run_host()
    main_r.stream.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main_r.stream)
    for _ in range(steps):
        main_r.run_host()
    e1.record(main_r.stream)
    e1.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / steps
    # one more plain run of each checked runner, then parity on rank 0's copy
    for name in ("fused", "fused_ordered", "nccl"):
        if name in runners:
            runners[name].run()
    torch.cuda.synchronize(device)
    dev_err = _lib.load().sf_q4_check_device_error()
    parity = {"tol": 1e-3, "checked": "all-reduced o and down outputs of the first and last layer, every row, "
                                      "vs fp64 product of the unsharded weights' fp32 dequant",
              "errors": {}}
    worst = 0.0
    for li in sorted({0, n_layers - 1}):
        for pi, which in ((3, 0), (6, 1)):
            name, n, k = shapes(workload)[pi]
            W, _ = _tp_weight(workload, li, pi, device, range(TP_BLOCKS))
            p, s_ = pack_weights_device(W, 128)
            del W
            wd = _dequant_ref(p, s_, 128).double()
            y_ref = _tp_x(li, pi, k, 1, device).double() @ wd.T
            del wd, p, s_
            for rn in ("fused", "fused_ordered", "nccl"):
                if rn not in runners:
                    continue
                y = runners[rn].red[li, which].double()
                err = ((y - y_ref).abs().max() / y_ref.abs().max()).item()
                parity["errors"][f"{rn}:L{li}.{name}"] = float(f"{err:.3e}")
                worst = max(worst, err)
    parity["max_err"] = float(f"{worst:.3e}")
    parity["ok"] = bool(worst <= 1e-3 and dev_err == 0)
    step_bytes = main_r.algorithmic_bytes()
    t = torch.tensor([times[k_] for k_ in sorted(times)] + [e2e_ms, float(not parity["ok"])],
                     device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    vals = t.tolist()
    times = dict(zip(sorted(times), vals[:len(times)]))
    e2e_ms = vals[len(times)]
    parity["ok_all_ranks"] = vals[-1] == 0.0
    peak, peak_kind = measured_peak()
    ms = times["fused"]
    per_gpu = step_bytes / (ms * 1e-3) / 1e9
    out = {
        "workload": f"BASELINE config 5: {workload}-shaped decode step, {n_layers} layers x 7 projections, "
                    f"sym int4 g128, bf16 activations, sharded over {world} GPU(s)",
        "parallelism": f"tp{world}: q/k/v/gate/up column-parallel, o/down row-parallel + all-reduce "
                       f"({2 * n_layers} per step)",
        "scaling": "strong",
        "n_gpus": world,
        "batch": 1,
        "fused_us": round(ms * 1e3, 1),
        "fused_ordered_us": round(times["fused_ordered"] * 1e3, 1),
        "fused_batch8_us": round(times["fused_batch8"] * 1e3, 1),
        "fused_no_exchange_us": round(times["fused_no_exchange"] * 1e3, 1) if "fused_no_exchange" in times else None,
        "peer_us": round(times["peer"] * 1e3, 1) if "peer" in times else None,
        "nccl_us": round(times["nccl"] * 1e3, 1) if "nccl" in times else None,
        "gbs_per_gpu": round(per_gpu, 1),
        "gbs_aggregate": round(per_gpu * world, 1),
        "bytes_per_gpu": step_bytes,
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "peak_kind": peak_kind,
                     "frac": round(per_gpu / peak, 4), "hbm_bound_us": round(step_bytes / peak / 1e3, 1),
                     "note": "whole fused step per GPU (GEMV streaming + in-kernel all-reduces)"},
        "e2e_us": round(e2e_ms * 1e3, 1),
        "parity": parity,
        "timing": f"CUDA events over {steps} graph replays per variant, max over ranks",
        "data": "seeded N(0,0.02) weights drawn in 8 blocks (the same matrix at every TP), RTN int4 on "
                "the device; bf16 N(0,1) inputs shared by every rank",
        "build_s": round(build_s, 1),
    }
    if dev_err != 0:
        out["device_error"] = dev_err
    del main_r
    # the caller prints its line first, then releases graphs and the communicator
    return out, (lambda: _teardown(dist, comm, runners, exit_dist=False))


def run_tp(args, rank, world, local_rank):
    """--workload 70b: the config-5 tensor-parallel step as its own JSON line."""
    import torch
    if args.layers and not args.tp_layers:
        args.tp_layers = args.layers
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)
    with ClockSampler(local_rank) as clocks:
        tp, cleanup = tp_measure(args, rank, world, local_rank, dist)
    if "unavailable" in tp:
        if rank == 0:
            print(json.dumps({"metric": "int4 GEMV HBM GB/s, 70b tensor-parallel decode step", **tp}))
        return
    total = tp["bytes_per_gpu"] * world
    result = {
        "metric": "int4 GEMV HBM GB/s, 70b tensor-parallel decode step (batch 1)",
        "value": round(total / tp["fused_us"] / 1e3, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tp["fused_us"] / 1e3, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights (u8 nibbles) x bf16 activations, exact int32 products, fp32 accumulate",
        "data": "synthetic: " + tp["data"],
        "config": {"workload": tp["workload"], "batch": 1, "parallelism": tp["parallelism"],
                   "l2": "weights >> L2 (no flush needed)"},
        "roofline": {**tp["roofline"], "unit": "GB/s", "traffic": None},
        "e2e": {"value": round(total / tp["e2e_us"] / 1e3, 1), "unit": "GB/s",
                "ms_per_step": round(tp["e2e_us"] / 1e3, 5), "h2d_bytes_per_step": None,
                "d2h_bytes_per_step": None,
                "api": "siliconfer_b200.tensor_parallel.TPStepRunner.run_host (pinned host in/out)"},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
        "tp70b": tp,
    }
    if rank == 0:
        print(json.dumps(result), flush=True)
    _exit_watchdog()
    cleanup()
    if dist is not None:
        dist.destroy_process_group()


def _exit_watchdog(seconds=60):
    """Ends the process if teardown blocks after the result line was printed."""
    def _force_exit():
        time.sleep(seconds)
        os._exit(0)
    threading.Thread(target=_force_exit, daemon=True).start()


def _teardown(dist, comm, runners, *refs, exit_dist=True):
    """Release captured graphs and the peer communicator (every rank together),
    then optionally the process group."""
    import gc
    import torch
    torch.cuda.synchronize()
    runners.clear()
    del refs
    gc.collect()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    if comm is not None:
        comm.close()
    if dist is not None:
        dist.barrier()
        if exit_dist:
            dist.destroy_process_group()


def _time_replays(replay, stream, n, flush=None):
    """Device time of one replay (ms), CUDA events on `stream`.  With `flush`
    (a buffer larger than L2) every replay is timed alone after the buffer
    was overwritten, so each one starts with cold caches."""
    import torch
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(n):
                replay()
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / n
    tot = 0.0
    for _ in range(n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            flush.add_(1)
            e0.record(stream)
            replay()
            e1.record(stream)
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / n


def sweep_measure(layers, device, args):
    """BASELINE config 3's batch sweep: the same 7B step at 4 and 16 tokens,
    each one launch that reads every weight once (batch 1 is the headline)."""
    import torch
    from siliconfer_b200.runner import Q4StepRunner
    peak, peak_kind = measured_peak()
    out = []
    for t in (4, 16):
        r = Q4StepRunner(layers, tokens=t, x_dtype=torch.float16, y_dtype=torch.float32, device=device,
                         waits=[False] * len(layers))
        g = torch.Generator(device=device)
        g.manual_seed(70 + t)
        r.x.copy_(torch.randn(r.x.shape, generator=g, device=device).to(r.x.dtype))
        r.capture()
        with torch.cuda.stream(r.stream):
            for _ in range(args.warmup):
                r.graph.replay()
            ms = _time_replays(r.graph.replay, r.stream, max(5, min(args.steps, 20)))
        nb = r.algorithmic_bytes()
        out.append({"batch": t, "us": round(ms * 1e3, 1), "gbs": round(nb / ms / 1e6, 1),
                    "frac": round(nb / ms / 1e6 / peak, 4), "bytes": nb, "launches_per_step": r.kernels_per_step})
        del r
    return {"workload": "BASELINE config 3 (7B step, sym int4 g128, fp16 x) at batch 4 and 16; one launch of "
                        "the decode kernel per step, every weight read once", "peak_gbs": peak,
            "peak_kind": peak_kind, "timing": "CUDA events over back-to-back graph replays (weights 3.44 GB >> L2)",
            "points": out}


def small_configs_measure(device, iters=20):
    """BASELINE configs 1 and 2 on Qwen2.5-0.5B shapes (hidden 896, inter 4864).

    config 1: one layer, sym RTN int4 g128, batch 1, fp32 x -- 7.9 MB, a latency figure;
    config 2: the 24-layer step, ASYMMETRIC int4 g128 with fp32 zeros (one 60-sigma outlier in
    layer 0's down_proj), batch 1, fp32 x.  The weights are quantized on the device with the
    reference's RTN (bit-exact); the HQQ grid choice (an offline quantizer) is not repeated here.
    Both are timed one replay at a time after overwriting a 256 MB buffer (L2 flushed)."""
    import torch
    from siliconfer_b200.q4_linear import Q4Linear
    from siliconfer_b200.quant import pack_weights_device
    from siliconfer_b200.runner import Q4StepRunner
    peak, _ = measured_peak()
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=device)   # 256 MB > L2
    out = {}
    for name, n_layers, sym in (("config1_0p5b_layer_sym", 1, True), ("config2_0p5b_24layers_asym", 24, False)):
        gen = torch.Generator(device=device)
        layers = []
        for li in range(n_layers):
            for pi, (pname, n, k) in enumerate(shapes("0.5b")):
                gen.manual_seed(5000 + 100 * li + pi)
                W = torch.randn((n, k), generator=gen, device=device) * 0.02
                if not sym and li == 0 and pname == "down":
                    W[17, 1234] = 60 * 0.02
                trip = pack_weights_device(W, 128, sym=sym)
                layers.append(Q4Linear(trip[0], trip[1], zeros=None if sym else trip[2], group_size=128,
                                       device=device))
        r = Q4StepRunner(layers, tokens=1, x_dtype=torch.float32, y_dtype=torch.float32, device=device,
                         waits=[False] * len(layers))
        r.x.normal_()
        r.capture()
        with torch.cuda.stream(r.stream):
            for _ in range(3):
                r.graph.replay()
        ms = _time_replays(r.graph.replay, r.stream, iters, flush=flush)
        nb = r.algorithmic_bytes()
        out[name] = {"layers": n_layers, "layout": "sym" if sym else "asym (fp32 zeros)", "us": round(ms * 1e3, 2),
                     "gbs": round(nb / ms / 1e6, 1), "frac": round(nb / ms / 1e6 / peak, 4), "bytes": nb,
                     "launches_per_step": r.kernels_per_step}
        del r, layers
    out["timing"] = "each replay timed alone with CUDA events after a 256 MB buffer write (cold L2)"
    return out


def per_call_measure(device, n=200):
    """The reference-shaped call: one Q4Linear forward per projection
    (siliconfer/model/q4_linear.py:49-68), on 7B q_proj (4096 x 4096, sym g128),
    batch 1.  `torch_*`: fp16 activation already on the GPU, output left on
    it (the module API: ctypes call, output allocation, pre-pass + GEMV
    launches); device time per call from CUDA events over n back-to-back
    calls, host time per call from the wall clock of the same loop.
    `numpy_us`: numpy fp32 in, numpy fp32 out (H2D copy, kernels, D2H copy,
    synchronisation), wall clock per call, like the reference's call."""
    import torch
    from siliconfer_b200.q4_linear import Q4Linear
    from siliconfer_b200.quant import pack_weights_device
    g = torch.Generator(device=device)
    g.manual_seed(11)
    p, sc = pack_weights_device(torch.randn((4096, 4096), generator=g, device=device) * 0.02, 128)
    m = Q4Linear(p, sc, group_size=128, device=device)
    x = torch.randn((1, 4096), generator=g, device=device).half()
    for _ in range(20):
        m(x)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(n):
        m(x)
    e1.record()
    host_us = (time.perf_counter() - t0) / n * 1e6
    e1.synchronize()
    dev_us = e0.elapsed_time(e1) / n * 1e3
    xn = x.float().cpu().numpy()
    for _ in range(10):
        m(xn)
    t0 = time.perf_counter()
    for _ in range(n // 4):
        m(xn)
    np_us = (time.perf_counter() - t0) / (n // 4) * 1e6
    nb = 4096 * 2048 + 4096 * 32 * 4 + 4096 * 2 + 4096 * 4
    return {"workload": "Q4Linear.forward on 7B q_proj (4096x4096, sym int4 g128), batch 1",
            "torch_device_us": round(dev_us, 2), "torch_host_us": round(host_us, 2),
            "torch_gbs": round(nb / dev_us / 1e3, 1), "numpy_us": round(np_us, 2),
            "kernels_per_call": 2}


def int2_measure(device, args):
    """2-bit weights (the reference's pack_int2 format, which it cannot serve)
    on the 7B step: 32 layers x 7 projections, symmetric, group 128, fp16 x,
    batch 1, one launch.  The 2-bit codes and the scales are drawn at random
    on the device (the kernel's speed does not depend on their values; its
    results are checked against the oracle in the tests)."""
    import torch
    from siliconfer_b200.q4_linear import Q4Linear
    from siliconfer_b200.runner import Q4StepRunner
    peak, peak_kind = measured_peak()
    gen = torch.Generator(device=device)
    gen.manual_seed(2)
    layers = []
    for _ in range(HIDDEN["7b"][2]):
        for _, n, k in shapes("7b"):
            p = torch.randint(0, 256, (n, k // 4), generator=gen, device=device, dtype=torch.uint8)
            sc = torch.rand((n, k // 128), generator=gen, device=device) * 0.01 + 0.005
            layers.append(Q4Linear(p, sc, group_size=128, device=device, bits=2))
    r = Q4StepRunner(layers, tokens=1, x_dtype=torch.float16, y_dtype=torch.float32, device=device,
                     waits=[False] * len(layers))
    r.x.normal_()
    r.capture()
    with torch.cuda.stream(r.stream):
        for _ in range(args.warmup):
            r.graph.replay()
    ms = _time_replays(r.graph.replay, r.stream, max(5, min(args.steps, 20)))
    nb = r.algorithmic_bytes()
    return {"workload": "7B step, 2-bit symmetric weights (pack_int2 layout), group 128, fp16 x, batch 1",
            "us": round(ms * 1e3, 1), "gbs": round(nb / ms / 1e6, 1), "frac": round(nb / ms / 1e6 / peak, 4),
            "peak_kind": peak_kind, "bytes": nb, "launches_per_step": r.kernels_per_step,
            "timing": "CUDA events over back-to-back graph replays (weights 1.8 GB >> L2)"}


def prefill_measure(device, stream, iters=20):
    """gemm_asym prefill at 7B shapes on the tcgen05 path.

    Asymmetric int4 g128 (device RTN), bf16 activations N(0,1), bf16 out.
    Each shape: warm-up on `stream`, then `iters` calls captured in a CUDA
    graph and timed with CUDA events around one replay (inputs stay resident;
    weights + X + Y of the largest shape are 61 MB, below L2, so this is the
    kernel's compute-bound speed with warm operands)."""
    import torch
    from siliconfer_b200 import quant as Q
    from siliconfer_b200.kernels import cuda as K
    peak, kind = 1590.0, "fallback bf16 burst (no MEASURED_PEAKS.json)"
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peak, kind = float(json.loads(pk.read_text())["bf16_tflops"]), "measured bf16 burst"
    out = []
    g = torch.Generator(device=device)
    for m in (512, 2048):
        for k, n in ((4096, 4096), (4096, 11008), (11008, 4096)):
            g.manual_seed(m + k + n)
            W = torch.randn((n, k), generator=g, device=device) * 0.02
            p, s, z = Q.pack_weights_device(W, 128, sym=False)
            del W
            X = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    K.linear(p, s, z, X, 128, out_dtype=torch.bfloat16)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(iters):
                    K.linear(p, s, z, X, 128, out_dtype=torch.bfloat16)
            with torch.cuda.stream(stream):
                graph.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                graph.replay()
                e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) / iters * 1e3
            tf = 2.0 * m * n * k / us / 1e6
            out.append({"M": m, "K": k, "N": n, "us": round(us, 1), "tflops": round(tf, 1),
                        "frac": None if peak is None else round(tf / peak, 4)})
            del graph, p, s, z, X
    return {"workload": "BASELINE config 4: gemm_asym prefill, 7B shapes, asym int4 g128, bf16 X",
            "kernel": "q4_gemm_tc_kernel (tcgen05, dequant to bf16 in TMEM)", "peak_tflops": peak,
            "peak_kind": kind, "shapes": out}


def kv_attention_measure(device, stream, iters=20):
    """Decode attention over the int8 KV cache (siliconfer's
    fused_quantized_attention_decode) at cache sizes above L2: HBM-bound,
    bytes = int8 K and V codes + fp32 scales (+ q, out)."""
    import torch
    from siliconfer_b200.kv_attention import fused_quantized_attention_decode, quantize_kv
    peak, _ = measured_peak()
    out = []
    g = torch.Generator(device=device)
    g.manual_seed(3)
    for B, H, Hkv, T, D in ((16, 64, 8, 8192, 128), (8, 32, 32, 4096, 128)):
        kc, ks = quantize_kv(torch.randn((B, Hkv, T, D), generator=g, device=device, dtype=torch.bfloat16))
        vc, vs = quantize_kv(torch.randn((B, Hkv, T, D), generator=g, device=device, dtype=torch.bfloat16))
        q = torch.randn((B, H, D), generator=g, device=device, dtype=torch.bfloat16)
        with torch.cuda.stream(stream):
            for _ in range(3):
                fused_quantized_attention_decode(q, kc, ks, vc, vs)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(iters):
                fused_quantized_attention_decode(q, kc, ks, vc, vs)
            e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) / iters * 1e3
        nbytes = 2 * B * Hkv * T * (D + 4) + B * H * D * 2 + B * H * D * 4
        out.append({"B": B, "H": H, "Hkv": Hkv, "T": T, "D": D, "us": round(us, 1),
                    "gbs": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / peak, 4)})
        del kc, ks, vc, vs, q
    return {"kernel": "kv_attn_tc_kernel + kv_attn_merge_kernel (int8 KV, mma.sync, fp32 online softmax; kv_attn_split_kernel only for head_dim 256)",
            "bound": "hbm", "peak_gbs": peak, "timing": "CUDA events around 20 back-to-back calls",
            "shapes": out}


def profile_prefill(m, k, n):
    """Three prefill GEMMs of one config-4 shape (asym int4 g128, bf16 X and Y)."""
    import torch
    from siliconfer_b200 import quant as Q
    from siliconfer_b200.kernels import cuda as K
    g = torch.Generator(device="cuda")
    g.manual_seed(m + k + n)
    W = torch.randn((n, k), generator=g, device="cuda") * 0.02
    p, s, z = Q.pack_weights_device(W, 128, sym=False)
    X = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        K.linear(p, s, z, X, 128, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    print(json.dumps({"profile_prefill": [m, k, n], "ok": True}))


def traffic_from_profile(workload, batch):
    """DRAM bytes per launch of the GEMV kernel, from the committed ncu summary
    (profiles/traffic.txt: lines "<workload>_b<batch> <bytes> <how>"), if any."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        f = line.split()
        if len(f) >= 2 and f[0] == f"{workload}_b{batch}":
            return int(f[1])
    return None


# ---------------------------------------------------------------------------
# CPU legs (reference's compiled kernels, else the oracle's C port)
# ---------------------------------------------------------------------------
def _cpu_impl():
    from oracle import cref
    if cref.ref_available():
        return cref.ref_gemm, "reference", "siliconfer q4_gemv_sym_neon (scalar C on x86) " \
                                           "compiled from the reference sources, rows split over threads"
    return cref.oracle_gemm, "port", "oracle C restatement, rows split over threads"


def _host_triples(workload, layers, n_layers_sample, batch):
    if layers is not None:
        trip = [(m.packed_d.cpu().numpy(), m.scales_d.cpu().numpy())
                for m in layers[:7 * n_layers_sample]]
    else:
        from siliconfer_b200.quant import pack_weights_sym
        rng = np.random.default_rng(1234)
        trip = []
        for _ in range(n_layers_sample):
            for _, n, k in shapes(workload):
                trip.append(pack_weights_sym(rng.normal(0, 0.02, (n, k)).astype(np.float32), 128))
    xs = [np.random.default_rng(i).normal(0, 1, (batch, p.shape[1] * 2)).astype(np.float16)
          .astype(np.float32) for i, (p, _) in enumerate(trip)]
    return trip, xs


def _time_cpu(trip, xs, batch, budget_s):
    fn, kind, desc = _cpu_impl()
    threads = os.cpu_count() or 1
    nbytes = sum(p.nbytes + s.nbytes + batch * (p.shape[1] * 2 * 4 + p.shape[0] * 4)
                 for p, s in trip)
    # one untimed pass, then as many passes as fit the budget
    t0 = time.perf_counter()
    for (p, s), x in zip(trip, xs):
        fn(p, s, None, x, 128, threads=threads)
    one = time.perf_counter() - t0
    reps = max(1, int(budget_s / max(one, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        for (p, s), x in zip(trip, xs):
            fn(p, s, None, x, 128, threads=threads)
    dt = (time.perf_counter() - t0) / reps
    return nbytes / dt / 1e9, dt, kind, desc, threads


def cpu_baseline(args, layers):
    n_sample = 2 if args.workload != "0.5b" else HIDDEN["0.5b"][2]
    trip, xs = _host_triples(args.workload, layers, n_sample, args.batch)
    gbs, dt, kind, desc, threads = _time_cpu(trip, xs, args.batch, budget_s=10.0)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{n_sample} of {HIDDEN[args.workload][2]} layers (7 projections each), "
                      f"batch {args.batch}: {dt * 1e3:.1f} ms per sample; {desc}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    n_sample = 2 if args.workload != "0.5b" else HIDDEN["0.5b"][2]
    trip, xs = _host_triples(args.workload, None, n_sample, args.batch)
    vals = []
    for _ in range(args.warmup):
        _time_cpu(trip, xs, args.batch, budget_s=0.0)
    for _ in range(args.steps):
        gbs, dt, kind, desc, threads = _time_cpu(trip, xs, args.batch, budget_s=0.0)
        vals.append((gbs, dt))
    gbs = statistics.median(v[0] for v in vals)
    dt = statistics.median(v[1] for v in vals)
    full_layers = HIDDEN[args.workload][2]
    print(json.dumps({
        "impl": "reference",
        "metric": f"int4 GEMV HBM GB/s, {args.workload} decode step (batch {args.batch})",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3 * full_layers / n_sample, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 weights x fp32 activations (fp16-representable), fp32 accumulate",
        "data": "synthetic: seeded N(0,0.02) weights, RTN int4 sym g128",
        "config": workload_config(args, world, HIDDEN[args.workload][2], "sym"),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{n_sample} of {full_layers} layers per step "
                                   f"(ms_per_step extrapolated to all layers); {desc}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="7b", choices=sorted(HIDDEN))
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill measurement")
    ap.add_argument("--profile-prefill", type=int, nargs=3, metavar=("M", "K", "N"),
                    help="run the config-4 prefill GEMM three times on one shape and exit (a profiling case)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers of the workload (default: all); smaller values are "
                         "profiling cases, not bench lines")
    ap.add_argument("--no-tp70b", action="store_true",
                    help="skip the config-5 tensor-parallel 70B step that the default line carries as 'tp70b'")
    ap.add_argument("--tp-layers", type=int, default=0,
                    help="decoder layers of the tp70b step (default: all 80); smaller values are "
                         "profiling cases, not bench lines")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.profile_prefill:
        profile_prefill(*args.profile_prefill)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    elif args.workload == "70b":
        run_tp(args, rank, world, local_rank)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
