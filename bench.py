#!/usr/bin/env python
"""Benchmark of the MMVQ hot path: the per-token quantized-GEMV chain of a decode model.

A "step" is one token's pass over the chain: every distinct input quantised to Q8_1
and every weight matrix multiplied once (the default workload, qwen3_8b: 253 GEMVs over
4.51 GB of Q4_K/Q6_K weights, 145 distinct inputs).  Weights are synthetic (seeded, drawn
on the GPU in GGUF block layout with the workload's value distributions) and far larger
than L2, so every step streams them from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                  [--executor persistent|graph] [--impl anvil|reference]

Executors: "graph" replays a CUDA graph of separate quantize + MMVQ launches with
programmatic dependent launch; "persistent" runs the token as one cooperative kernel (groups
of GEMVs sharing an input, Q8_1 quantisation inside the kernel, a grid barrier before each
group that depends on earlier ones).  The default, "auto", takes the graph on one GPU and
the persistent kernel on several (no collective library in the data path).

One JSON line is printed by rank 0:
  value        chain bytes / device time, whole job (GB/s): weights + Q8_1 reads + fp32
               outputs, timed with CUDA events around K launches, max over ranks
  e2e          the same metric through the public API with the step's fp32 inputs copied
               host->device from pinned memory and the logits copied back, every step
  roofline     the dominant kernel: algorithmic bytes per launch / average launch time
               measured here with CUDA events, against measured HBM copy bandwidth
  cpu_baseline the CPU oracle (oracle/, all host threads) on a bounded sample of the same
               workload (layer 0 of the chain), rank 0 at N=1 only
With N > 1 (torchrun), --multi replicas (default) runs one full chain per GPU on its own
inputs: independent token streams, no collective in the data path, weak scaling (the
8B-class workloads fit one GPU).  --multi rows shards every matrix by rows across the GPUs
(strong scaling): the persistent executor writes each output row into every rank's output
buffer over NVLink (CUDA IPC peer stores) inside the kernel; the graph executor
all-gathers each GEMV's output with NCCL inside the CUDA graph.
--impl reference times the CPU oracle port on the same workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "kernel-anvil_b200", ROOT):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "Q4_K GEMV weight-stream GB/s (% of HBM peak); per-token GEMV-chain µs"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="qwen3_8b")
    ap.add_argument("--gemvs", type=int, default=0,
                    help="only the workload's first N GEMVs (a smaller case of the same shapes)")
    ap.add_argument("--impl", default="anvil", choices=["anvil", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quantize", choices=["fused", "separate"], default="separate",
                    help="quantise each GEMV input in its own kernel or inside the GEMV (fused)")
    ap.add_argument("--coresident", type=int, default=1,
                    help="graph executor: GEMV kernels sized to share each SM")
    ap.add_argument("--executor", choices=["auto", "persistent", "graph"], default="auto",
                    help="one persistent kernel per token, or a CUDA graph of per-GEMV launches "
                         "(auto: graph on one GPU, persistent with peer stores on several)")
    ap.add_argument("--grouped", type=int, default=1,
                    help="graph executor: one launch per run of same-type GEMVs on one input (1) "
                         "quantising in the kernel, or one launch per GEMV (0)")
    ap.add_argument("--glu", type=int, default=0,
                    help="grouped graph executor: each layer's ffn_gate/ffn_up pair as one launch "
                         "with silu(gate) * up in the epilogue (1), or as a grouped GEMV pair (0)")
    ap.add_argument("--multi", choices=["replicas", "rows"], default="replicas",
                    help="N > 1: one full chain per GPU (independent token streams, no collective; "
                         "weak scaling) or every matrix row-sharded across the GPUs with the outputs "
                         "exchanged (strong scaling)")
    ap.add_argument("--nwarps", type=int, default=0, help="persistent executor: warps per CTA (0 = 8)")
    ap.add_argument("--ctas-per-sm", type=int, default=0, help="persistent executor: CTAs per SM (0 = 1)")
    return ap.parse_args()


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) across the timed region: SM clocks and throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        return self

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        rows = [ln.split(", ") for ln in Path(self.out.name).read_text().splitlines() if ln.strip()]
        os.unlink(self.out.name)
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = max(smax, float(r[2]))
                for name, flag in zip(names, r[5:9]):
                    if flag.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle on layer 0 of the workload
# ---------------------------------------------------------------------------------------

def cpu_sample(workload: str):
    """Layer 0 (or the first 7 GEMVs) of the chain, generated on the host."""
    from kernel_anvil.chains import get_chain
    from kernel_anvil.quants import gemv_bytes, make_activation, make_weights

    spec = get_chain(workload)
    gemvs = [g for g in spec.gemvs if g.name.startswith("blk.0.")] or spec.gemvs[:7]
    inputs = {}
    for g in gemvs:
        inputs.setdefault(g.input, g.K)
    W = [make_weights(g.qt, g.nrows, g.K, seed=i) for i, g in enumerate(gemvs)]
    x = {a: make_activation(k, seed=j) for j, (a, k) in enumerate(inputs.items())}
    nbytes = sum(gemv_bytes(g.qt, g.nrows, g.K) for g in gemvs)
    desc = f"{workload} layer 0: {len(gemvs)} GEMVs + {len(inputs)} quantisations, {nbytes/1e6:.1f} MB"
    return gemvs, W, x, nbytes, desc


def cpu_step(gemvs, W, x):
    from oracle import oracle

    xq = {a: oracle.quantize_q8_1(v) for a, v in x.items()}
    for g, w in zip(gemvs, W):
        oracle.mmvq(g.qt, w, xq[g.input], g.nrows, g.K)


def use_all_host_threads() -> None:
    """The oracle's OpenMP team = every core this process may run on.  torchrun sets
    OMP_NUM_THREADS=1 in its workers, which would otherwise time the CPU leg on one core."""
    from oracle import oracle

    oracle.set_num_threads(len(os.sched_getaffinity(0)))


def cpu_baseline(workload: str, seconds: float) -> dict:
    from oracle import oracle

    use_all_host_threads()
    gemvs, W, x, nbytes, desc = cpu_sample(workload)
    cpu_step(gemvs, W, x)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_step(gemvs, W, x)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": round(nbytes * reps / dt / 1e9, 3), "unit": "GB/s", "cores": oracle.num_threads(),
            "kind": "port", "sample": f"{desc}; {reps} passes in {dt:.1f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle

    use_all_host_threads()
    gemvs, W, x, nbytes, desc = cpu_sample(args.workload)
    for _ in range(args.warmup):
        cpu_step(gemvs, W, x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(gemvs, W, x)
    dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 dp4a / fp32", "data": "synthetic",
        "config": {"workload": f"{args.workload} (CPU sample: layer 0)", "sample": desc},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": oracle.num_threads(),
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------

def time_graph(launch, stream, steps: int) -> float:
    """Milliseconds per launch over `steps` launches, CUDA events on `stream`."""
    import torch

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        launch()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def dominant_kernel(dc, stream, steps: int, warmup: int) -> dict:
    """The Q4_K MMVQ launches of one chain step, launched as in the chain (one launch per
    run of Q4_K GEMVs on one input when grouped) and replayed as their own PDL graph."""
    import torch

    from kernel_anvil.chains import is_gate_up
    from kernel_anvil.mmvq import Chain, q8_1_bytes
    from kernel_anvil.quants import gemv_bytes

    ch = Chain()
    nbytes, n = 0, 0
    gemvs = list(zip(dc.spec.gemvs, dc.weights, dc.outputs, dc.rows))
    i = 0
    while i < len(gemvs):
        gm = gemvs[i][0]
        j = i + 1
        if dc.grouped:
            while (j < len(gemvs) and j - i < 4 and gemvs[j][0].input == gm.input
                   and gemvs[j][0].qt == gm.qt):
                j += 1
        if gm.qt == "Q4_K" and dc.glu and is_gate_up([g for g, _, _, _ in gemvs[i:j]]):
            ch.add_mmvq_glu(gemvs[i][1], gemvs[i + 1][1], gm.qt, dc.xq[gm.input], gemvs[i][2])
            r = gemvs[i][3][1] - gemvs[i][3][0]
            nbytes += 2 * gemv_bytes(gm.qt, r, gm.K, 1) - 4 * r - q8_1_bytes(gm.K)
            n += 1
        elif gm.qt == "Q4_K":
            run = gemvs[i:j]
            rows = [r1 - r0 for _, _, _, (r0, r1) in run]
            ch.add_mmvq_grouped([w for _, w, _, _ in run], gm.qt, dc.xq[gm.input],
                                [y for _, _, y, _ in run], rows, K=gm.K, ncols=dc.ncols)
            nbytes += sum(gemv_bytes(gm.qt, r, gm.K, dc.ncols) for r in rows)
            n += 1
        i = j
    with torch.cuda.stream(stream):
        ch.instantiate(pdl=True)
        for _ in range(warmup):
            ch.launch()
        ms = time_graph(ch.launch, stream, steps)
    ch.close()
    return {"launches_per_step": n, "bytes_per_launch": nbytes / n, "ms_per_launch": ms / n}


def traffic_per_launch(kernel: str) -> float | None:
    """dram read+write bytes per launch of `kernel` from the committed ncu summaries (a line
    `<kernel> dram_bytes_per_launch: N`); None when not captured."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        try:
            for line in p.read_text().splitlines():
                if line.startswith(f"{kernel} dram_bytes_per_launch:"):
                    return float(line.split(":", 1)[1])
        except OSError:
            pass
    return None


def run_anvil(args) -> None:
    import torch
    import torch.distributed as dist

    from kernel_anvil import mmvq as ops
    from kernel_anvil.chains import DeviceChain, get_chain

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    spec = get_chain(args.workload)
    if args.gemvs:
        spec = spec.head(args.gemvs)
    shard = world > 1 and args.multi == "rows"
    if args.executor == "auto":
        args.executor = "persistent" if shard else "graph"
    persistent = args.executor == "persistent"
    # replicas: every rank runs the whole chain on its own inputs (seeded per rank)
    dc = DeviceChain(spec, rank=rank if shard else 0, world=world if shard else 1, device=dev,
                     seed=0 if shard else rank, fused=args.quantize == "fused",
                     coresident=args.coresident, executor=args.executor,
                     dist=dist if shard else None, nwarps=args.nwarps,
                     ctas_per_sm=args.ctas_per_sm, grouped=bool(args.grouped) and not persistent,
                     glu=bool(args.glu))
    stream = torch.cuda.Stream(device=dev)
    hbm_peak, peak_kind = measured_peaks()
    # whole job (gate/up launches write one vector per pair: the chain's own count)
    total_bytes = ((dc.algorithmic_bytes if dc.glu else spec.algorithmic_bytes())
                   * (1 if shard or world == 1 else world))
    rank_bytes = dc.algorithmic_bytes       # this rank's shard

    graph = None
    launches_per_step = dc.launches_per_step
    n_quantize = dc.chain.n_quantize if dc.chain else 0
    if not shard or persistent:
        with torch.cuda.stream(stream):
            dc.instantiate(pdl=True)
        launch = dc.launch
    else:
        from kernel_anvil.sharded import ShardedStep
        step = ShardedStep(dc, dist)
        with torch.cuda.stream(stream):
            step.eager()  # warms NCCL before capture
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step.eager()
        launch = graph.replay

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-timed chain -------------------------------------------------------------
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            launch()
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local).start()
    with torch.cuda.stream(stream):
        ms = time_graph(launch, stream, args.steps)
    clk = clocks.stop()
    torch.cuda.synchronize()
    barrier()
    ms_rank = ms
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = total_bytes / (ms * 1e-3) / 1e9

    # ---- end to end: host inputs in, logits out, every step --------------------------------
    h_in = torch.empty(dc.x_all.numel(), dtype=torch.float32, pin_memory=True)
    h_in.copy_(dc.x_all.cpu())
    logits = dc.outputs[-1]
    h_out = torch.empty(logits.numel(), dtype=torch.float32, pin_memory=True)

    def e2e_step():
        dc.x_all.copy_(h_in, non_blocking=True)
        launch()
        h_out.copy_(logits.view(-1), non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(2):
            e2e_step()
    stream.synchronize()
    barrier()
    with torch.cuda.stream(stream):
        ms_e2e = time_graph(e2e_step, stream, args.steps)
    barrier()
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = {"value": round(total_bytes / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h_in.numel() * 4, "d2h_bytes_per_step": h_out.numel() * 4,
           "ms_per_step": round(ms_e2e, 4)}

    # ---- dominant kernel roofline -----------------------------------------------------------
    peak_source = (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                   else "fallback 6.65 TB/s")
    if persistent:
        # one launch per token: the kernel is the step; this rank's bytes over its time
        achieved = rank_bytes / (ms_rank * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(achieved / hbm_peak, 4),
                    "traffic": traffic_per_launch(f"pchain_kernel {args.workload}"),
                    "peak_source": peak_source,
                    "kernel": f"pchain_kernel<ncols={dc.ncols}> (whole token, one cooperative launch)",
                    "launches_per_step": 1, "bytes_per_launch": rank_bytes,
                    "us_per_launch": round(ms_rank * 1e3, 3)}
    else:
        dk = dominant_kernel(dc, stream, args.steps, args.warmup)
        achieved = dk["bytes_per_launch"] / (dk["ms_per_launch"] * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(achieved / hbm_peak, 4),
                    "traffic": traffic_per_launch(f"mmvq_kernel {args.workload}"),
                    "peak_source": peak_source,
                    "kernel": "mmvq_kernel<Q4_K, ncols=1> (all Q4_K launches of one step, PDL graph)",
                    "launches_per_step": dk["launches_per_step"],
                    "bytes_per_launch": round(dk["bytes_per_launch"]),
                    "us_per_launch": round(dk["ms_per_launch"] * 1e3, 3)}

    status = ops.take_device_status()
    pinfo, n_groups = None, 0
    if persistent:
        from kernel_anvil.pchain import take_status
        status |= take_status()
        pinfo = dc.pchain.info()
        n_groups = dc.pchain.n_groups
    if graph is not None:
        # the graph holds NCCL work: release it before the process group goes away
        launch = e2e_step = None
        graph.reset()
        del graph
    dc.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong" if shard or world == 1 else "weak",
        "vs_baseline": None,
        "dtype": "int8 dp4a / fp32", "data": "synthetic",
        "config": {"workload": f"{args.workload} per-token GEMV chain",
                   "gemvs_per_step": len(spec.gemvs),
                   "quantizations_per_step": n_groups if persistent else n_quantize,
                   "bytes_per_step": total_bytes, "weight_bytes": spec.weight_bytes(),
                   "us_per_token": round(ms * 1e3, 1), "pct_of_hbm_peak": round(100 * value / hbm_peak, 1),
                   "pct_of_8TBps": round(100 * value / 8000.0, 1),
                   "l2": "inputs larger than L2 (weights stream from HBM every step)",
                   "parallelism": ((f"row-shard x{world}, " + ("outputs written to every rank over NVLink "
                                    "(CUDA IPC peer stores) inside the kernel" if persistent else
                                    "NCCL all-gather per GEMV")) if shard else
                                   f"{world} replicas: one full chain per GPU on its own inputs, no "
                                   "collective in the data path" if world > 1 else "single GPU"),
                   "executor": ("one persistent cooperative kernel per token: groups of GEMVs sharing an "
                                "input, Q8_1 quantisation in-kernel, grid barrier between dependent groups"
                                if persistent else
                                "CUDA graph of quantize + MMVQ launches, programmatic dependent launch"),
                   "quantize": "in-kernel per group" if persistent else args.quantize,
                   "grouped_launches": bool(args.grouped) and not persistent,
                   "gate_up_glu": dc.glu,
                   **({"persistent": pinfo} if persistent else
                      {"coresident_kernels_per_sm": args.coresident})},
        "e2e": e2e, "roofline": roofline, "gpu_launches": launches_per_step * args.steps,
        "device_status": status,
    }
    if clk is not None:
        line["clocks"] = clk
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, args.cpu_seconds)
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_anvil(args)


if __name__ == "__main__":
    main()
