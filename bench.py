#!/usr/bin/env python
"""Benchmark of the MMVQ hot path: the per-token quantized-GEMV chain of a decode model.

A "step" is one token's pass over the chain: every GEMV input quantised to Q8_1 and every
weight matrix multiplied once.  The default workload is the Llama-3-70B-shaped Q4_K chain
(80 layers, 560 GEMVs over 38.5 GB of weights), every matrix row-sharded across the N GPUs
(N = 1 included: one shard is the whole matrix), run by the persistent executor: one
cooperative kernel per token per GPU, each group of GEMVs reading the previous group's
gathered output as it arrives (gate/up pairs as one gate/up GEMV with silu(gate) * up),
each GPU writing its output rows into every GPU's buffer over NVLink inside the kernel.
Weights are synthetic (seeded, drawn on the GPU in GGUF block layout with the workload's
value distributions) and far larger than L2, so every step streams them from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                  [--multi rows|replicas] [--executor persistent|graph] [--impl anvil|reference]

One JSON line is printed by rank 0:
  value        whole-job chain bytes / device time (GB/s): weights of all shards + Q8_1
               reads + fp32 outputs, timed with CUDA events around K launches, max over ranks
  e2e          the same metric through the public API with the step's external input (the
               token's fp32 embedding) copied host->device from pinned memory and the last
               output copied back, every step
  roofline     the dominant kernel (the persistent chain kernel: the whole step on each GPU):
               this GPU's algorithmic bytes per launch / its launch time, against the
               measured HBM copy bandwidth
  cpu_baseline the CPU oracle (oracle/, all host threads) on a bounded sample of the same
               workload (layer 0 of the chain), rank 0 at N=1 only, plus the reference's
               dependency path (gguf-py dequantize + numpy fp32 matvec) on one matrix
  extras       (N=1) the single Q4_K 4096 x 4096 GEMV and the Qwen3-8B chain in the same run
--multi replicas runs one full chain per GPU on its own inputs instead (no collective;
weak scaling).  --executor graph runs a CUDA graph of quantize + MMVQ launches on fixed
inputs (with --multi rows, an NCCL all-gather after every GEMV inside the graph).
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
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="llama3_70b")
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
                    help="one persistent kernel per token (the chain's data flow inside it), a CUDA "
                         "graph of quantize + MMVQ launches on fixed inputs, or auto: the graph on one "
                         "GPU (the faster single-GPU executor), the persistent kernel on several (its "
                         "in-kernel exchange of the row-sharded outputs)")
    ap.add_argument("--fixed-inputs", action="store_true",
                    help="persistent executor: every group reads a fixed synthetic input instead of "
                         "its producer's output")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the N=1 extra measurements (single 4096^2 GEMV, Qwen3-8B chain)")
    ap.add_argument("--trace", action="store_true",
                    help="persistent executor: record per-group timestamps of one extra launch")
    ap.add_argument("--grouped", type=int, default=1,
                    help="graph executor: one launch per run of same-type GEMVs on one input (1) "
                         "quantising in the kernel, or one launch per GEMV (0)")
    ap.add_argument("--glu", type=int, default=0,
                    help="grouped graph executor: each layer's ffn_gate/ffn_up pair as one launch "
                         "with silu(gate) * up in the epilogue (1), or as a grouped GEMV pair (0)")
    ap.add_argument("--multi", choices=["replicas", "rows"], default="rows",
                    help="every matrix row-sharded across the GPUs with the outputs exchanged (strong "
                         "scaling), or one full chain per GPU on its own inputs (no collective; weak "
                         "scaling)")
    ap.add_argument("--nwarps", type=int, default=0, help="persistent executor: warps per CTA (0 = 8)")
    ap.add_argument("--ctas-per-sm", type=int, default=0, help="persistent executor: CTAs per SM (0 = 1)")
    ap.add_argument("--smithy", default="auto",
                    help="launch-shape table for the MMVQ launches: auto (the table tuned on a B200 for "
                         "the workload, kernel_anvil/tuned/<workload>_b200.json, when there is one), "
                         "none (the built-in shapes), or a smithy JSON path; loaded through the same "
                         "loader llama.cpp's lookup uses")
    ap.add_argument("--ncols", type=int, default=1,
                    help="activation columns per step (speculative-decode verification batch; the "
                         "persistent executor takes 1 or 2, the graph executor 1..8)")
    ap.add_argument("--static-share", type=int, default=None,
                    help="persistent executor: percent of each group's tiles dealt round-robin, the "
                         "rest claimed at run time (default: the library's)")
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


def reference_dependency(workload: str, seconds: float = 4.0) -> dict:
    """The reference's dependency path on one matrix of the workload: gguf-py (gguf 0.19.0,
    kernel-anvil pyproject.toml:19) gguf.quants.dequantize of the GGUF blocks, then a numpy
    fp32 matvec with the Q8_1-dequantised activation.  Single-threaded numpy, as it runs."""
    import numpy as np
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    from kernel_anvil.chains import get_chain
    from kernel_anvil.quants import gemv_bytes, make_activation, make_weights
    from oracle import oracle

    spec = get_chain(workload)
    g = next((g for g in spec.gemvs if g.name.endswith("attn_k")), spec.gemvs[0])
    W = make_weights(g.qt, g.nrows, g.K, seed=1)
    x = oracle.dequantize_q8_1(oracle.quantize_q8_1(make_activation(g.K, seed=2)), g.K)[0]
    qtype = getattr(GGMLQuantizationType, g.qt)

    def one():
        Wf = dequantize(W.reshape(-1), qtype).reshape(g.nrows, g.K)
        return Wf @ x

    one()
    reps, t0 = 0, time.perf_counter()
    while True:
        one()
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    nbytes = gemv_bytes(g.qt, g.nrows, g.K)
    return {"value": round(nbytes * reps / dt / 1e9, 4), "unit": "GB/s", "cores": 1,
            "kind": "reference-dependency",
            "sample": f"{g.name} ({g.qt} {g.nrows}x{g.K}): gguf.quants.dequantize + numpy fp32 matvec, "
                      f"{reps} passes in {dt:.1f} s"}


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
    """Graph executor: the MMVQ launches of the chain's dominant weight type (the most weight
    bytes) in one step, launched as in the chain (one launch per run of that type's GEMVs on
    one input when grouped) and replayed as their own PDL graph."""
    import torch

    from kernel_anvil.chains import is_gate_up
    from kernel_anvil.mmvq import Chain, q8_1_bytes
    from kernel_anvil.quants import gemv_bytes, resolve_type

    by_type: dict = {}
    for g in dc.spec.gemvs:
        by_type[g.qt] = by_type.get(g.qt, 0) + g.nrows * resolve_type(g.qt).row_bytes(g.K)
    qt_dom = max(by_type, key=by_type.get)

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
        if gm.qt == qt_dom and dc.glu and is_gate_up([g for g, _, _, _ in gemvs[i:j]]):
            ch.add_mmvq_glu(gemvs[i][1], gemvs[i + 1][1], gm.qt, dc.xq[gm.input], gemvs[i][2])
            r = gemvs[i][3][1] - gemvs[i][3][0]
            nbytes += 2 * gemv_bytes(gm.qt, r, gm.K, 1) - 4 * r - q8_1_bytes(gm.K)
            n += 1
        elif gm.qt == qt_dom:
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
    return {"launches_per_step": n, "bytes_per_launch": nbytes / n, "ms_per_launch": ms / n,
            "qt": qt_dom}


def traffic_per_launch(kernel: str) -> tuple[float | None, str | None]:
    """DRAM read+write bytes per launch of `kernel` from the committed ncu summaries (a line
    `<kernel> dram_bytes_per_launch: N` with a following `<kernel> traffic_source: ...`);
    (None, None) when not captured."""
    val, src = None, None
    for p in sorted((ROOT / "profiles").glob("*.md")):
        try:
            for line in p.read_text().splitlines():
                if line.startswith(f"{kernel} dram_bytes_per_launch:"):
                    val = float(line.split(":", 1)[1])
                    src = f"profiles/{p.name}"
                elif line.startswith(f"{kernel} traffic_source:") and val is not None:
                    src = f"profiles/{p.name}: " + line.split(":", 1)[1].strip()
        except OSError:
            pass
        if val is not None:
            return val, src
    return None, None


def extra_config0(hbm_peak: float) -> dict:
    """The single Q4_K GEMV of N = K = 4096 (9,458,176 algorithmic bytes): per-GEMV time over
    a rotation of distinct weight copies (more bytes than L2), three ways: separate launches
    in a CUDA graph, the same with programmatic dependent launch, and 64 independent GEMVs
    run by one persistent kernel."""
    import torch

    from kernel_anvil.pchain import PersistentChain
    from kernel_anvil.verify import GemvBench

    out = {"shape": "Q4_K 4096x4096, 1 column", "bytes": None}
    for pdl in (False, True):
        b = GemvBench("Q4_K", 4096, 4096, pdl=pdl)
        us = b.time(warmup=64, runs=640)
        out["bytes"] = b.bytes
        out["pdl_launches_us" if pdl else "launches_us"] = round(us, 3)
        if not pdl:
            copies, W, x = b.copies, list(b.W), b.x
        b.close()
    pc = PersistentChain()
    for i in range(copies):
        pc.add_group(x)
        pc.add_gemv(W[i], "Q4_K", nrows=4096)
    pc.instantiate()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(3):
            pc.launch(stream)
        ms = time_graph(lambda: pc.launch(stream), stream, 20)
    pc.close()
    out["persistent_us"] = round(ms * 1e3 / copies, 3)
    out["gemvs_per_persistent_launch"] = copies
    for k in ("launches_us", "pdl_launches_us", "persistent_us"):
        gbs = out["bytes"] / (out[k] * 1e-6) / 1e9
        out[k.replace("_us", "_gbs")] = round(gbs, 1)
        out[k.replace("_us", "_pct_of_hbm_peak")] = round(100 * gbs / hbm_peak, 1)
        out[k.replace("_us", "_pct_of_8TBps")] = round(100 * gbs / 8000, 1)
    out["l2"] = f"{copies} distinct weight copies per rotation ({copies * 9437184 / 1e6:.0f} MB > L2)"
    return out


def extra_qwen3_8b(stream, steps: int, warmup: int) -> dict:
    """Config 1, the Qwen3-8B chain on this GPU: the persistent dataflow executor and the
    CUDA graph of grouped quantize + MMVQ launches on fixed inputs."""
    import torch

    from kernel_anvil.chains import DeviceChain, get_chain

    spec = get_chain("qwen3_8b")
    res = {"gemvs_per_step": len(spec.gemvs)}
    for name, kw in (("persistent_dataflow", {"executor": "persistent"}),
                     ("graph_fixed_inputs", {"executor": "graph", "grouped": True})):
        dc = DeviceChain(spec, **kw)
        with torch.cuda.stream(stream):
            dc.instantiate(pdl=True)
            for _ in range(max(warmup, 3)):
                dc.launch()
            ms = time_graph(dc.launch, stream, steps)
        nbytes = spec.glu_algorithmic_bytes() if dc.pchain else spec.algorithmic_bytes()
        res[name] = {"us_per_token": round(ms * 1e3, 1), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                     "launches_per_step": dc.launches_per_step}
        dc.close()
        del dc
        torch.cuda.empty_cache()
    return res


def load_launch_table(choice: str, workload: str) -> str | None:
    """Load the smithy table that sets the MMVQ launch shapes (anvil_smithy_load, the loader
    behind llama.cpp's lookup): the B200-tuned table of the workload for "auto", none for
    "none", else the given file.  Returns the file's name, or None when no table is active."""
    from kernel_anvil import _native

    lib = _native.lib()
    lib.anvil_smithy_reset()
    if choice == "none":
        return None
    path = (ROOT / "kernel-anvil_b200" / "kernel_anvil" / "tuned" / f"{workload}_b200.json"
            if choice == "auto" else Path(choice))
    if not path.exists():
        if choice != "auto":
            raise SystemExit(f"--smithy {choice}: no such file")
        return None
    n = lib.anvil_smithy_load(str(path).encode())
    if n <= 0:
        raise SystemExit(f"--smithy: {path} holds no usable cell ({n})")
    return f"{path.name} ({n} cells)"


def extra_persistent(spec, stream, steps: int, warmup: int) -> dict:
    """The headline chain on this GPU through the persistent dataflow executor (the executor
    of the row-sharded multi-GPU runs): its one-GPU time, for scaling comparisons."""
    import torch

    from kernel_anvil.chains import DeviceChain

    dc = DeviceChain(spec, executor="persistent")
    with torch.cuda.stream(stream):
        dc.instantiate(pdl=True)
        for _ in range(max(warmup, 3)):
            dc.launch()
        ms = time_graph(dc.launch, stream, steps)
    nbytes = spec.glu_algorithmic_bytes()
    res = {"us_per_token": round(ms * 1e3, 1), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
           "launches_per_step": 1, "groups_per_step": dc.pchain.info()["groups"]}
    dc.close()
    del dc
    torch.cuda.empty_cache()
    return res


def run_anvil(args) -> None:
    import torch
    import torch.distributed as dist

    from kernel_anvil import mmvq as ops
    from kernel_anvil.chains import DeviceChain, get_chain
    from kernel_anvil.pchain import take_status

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
    smithy = load_launch_table(args.smithy, args.workload)
    shard = args.multi == "rows"
    if args.executor == "auto":
        args.executor = "graph" if world == 1 or not shard else "persistent"
    persistent = args.executor == "persistent"
    # replicas: every rank runs the whole chain on its own inputs (seeded per rank)
    dc = DeviceChain(spec, rank=rank if shard else 0, world=world if shard else 1, device=dev,
                     seed=0 if shard else rank, fused=args.quantize == "fused",
                     coresident=args.coresident, executor=args.executor,
                     dist=dist if shard and world > 1 else None, nwarps=args.nwarps,
                     ctas_per_sm=args.ctas_per_sm, grouped=bool(args.grouped) and not persistent,
                     glu=bool(args.glu), dataflow=not args.fixed_inputs,
                     static_share=args.static_share, ncols=args.ncols)
    stream = torch.cuda.Stream(device=dev)
    hbm_peak, peak_kind = measured_peaks()
    # whole job: the unsharded chain once (shards), or every replica's chain
    one_chain = (spec.glu_algorithmic_bytes(args.ncols) if (persistent or dc.glu)
                 else spec.algorithmic_bytes(args.ncols))
    total_bytes = one_chain * (1 if shard else world)
    rank_bytes = dc.algorithmic_bytes       # this rank's launches

    graph = None
    launches_per_step = dc.launches_per_step
    n_quantize = dc.chain.n_quantize if dc.chain else 0
    if persistent or not (shard and world > 1):
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

    # ---- per-group trace of one more launch (persistent executor) ----------------------------
    trace = None
    if persistent and args.trace:
        from kernel_anvil.pchain import trace_summary
        tbuf = dc.pchain.enable_trace()
        with torch.cuda.stream(stream):
            launch()
        stream.synchronize()
        trace = trace_summary(tbuf)
        barrier()

    # ---- end to end: host input in, last output out, every step -----------------------------
    ext = dc.external_inputs
    xin = [dc.x[a] for a in ext]
    h_in = [torch.empty(x.numel(), dtype=torch.float32, pin_memory=True) for x in xin]
    for h, x in zip(h_in, xin):
        h.copy_(x.reshape(-1).cpu())
    if persistent:
        last = torch.empty((dc.ncols, spec.gemvs[-1].nrows), dtype=torch.float32, device=dev)

        def read_last():
            return dc.pchain.output(dc.pidx[-1], out=last, stream=stream)
    else:
        last = dc.outputs[-1]

        def read_last():
            return last
    h_out = torch.empty(last.numel(), dtype=torch.float32, pin_memory=True)

    def e2e_step():
        for h, x in zip(h_in, xin):
            x.view(-1).copy_(h, non_blocking=True)
        launch()
        h_out.copy_(read_last().view(-1), non_blocking=True)

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
           "h2d_bytes_per_step": sum(h.numel() for h in h_in) * 4, "d2h_bytes_per_step": h_out.numel() * 4,
           "ms_per_step": round(ms_e2e, 4), "us_per_token": round(ms_e2e * 1e3, 1)}

    # ---- dominant kernel roofline -----------------------------------------------------------
    peak_source = (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                   else "fallback 6.65 TB/s")
    if persistent:
        # one launch per token: the kernel is the step; this rank's bytes over its own time
        achieved = rank_bytes / (ms_rank * 1e-3) / 1e9
        traffic, tsrc = traffic_per_launch(f"pchain_kernel {args.workload} x{world}")
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "traffic_source": tsrc,
                    "peak_source": peak_source,
                    "kernel": f"pchain_kernel<ncols={dc.ncols}> (whole token, one cooperative launch per GPU)",
                    "launches_per_step": 1, "bytes_per_launch": rank_bytes,
                    "us_per_launch": round(ms_rank * 1e3, 3)}
    else:
        dk = dominant_kernel(dc, stream, args.steps, args.warmup)
        achieved = dk["bytes_per_launch"] / (dk["ms_per_launch"] * 1e-3) / 1e9
        traffic, tsrc = traffic_per_launch(f"mmvq_kernel {args.workload}")
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "traffic_source": tsrc,
                    "peak_source": peak_source,
                    "kernel": f"mmvq_kernel<{dk['qt']}, ncols={dc.ncols}> (all {dk['qt']} launches of "
                              "one step, PDL graph)",
                    "launches_per_step": dk["launches_per_step"],
                    "bytes_per_launch": round(dk["bytes_per_launch"]),
                    "us_per_launch": round(dk["ms_per_launch"] * 1e3, 3)}

    status = ops.take_device_status()
    pinfo, n_groups, dataflow = None, 0, dc.dataflow
    if persistent:
        status |= take_status()
        pinfo = dc.pchain.info()
        pinfo["static_share_pct"] = args.static_share if args.static_share is not None else "default"
        n_groups = pinfo["groups"]
    if graph is not None:
        # the graph holds NCCL work: release it before the process group goes away
        launch = e2e_step = None
        graph.reset()
        del graph
    dc.close()
    del dc
    torch.cuda.empty_cache()

    extras = {}
    if world == 1 and not args.no_extras:
        extras["config0_single_gemv"] = extra_config0(hbm_peak)
        extras["config1_qwen3_8b_chain"] = extra_qwen3_8b(stream, args.steps, args.warmup)
        if not persistent:
            extras["persistent_dataflow_same_chain"] = extra_persistent(spec, stream, args.steps,
                                                                        args.warmup)
        status |= ops.take_device_status() | take_status()

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    if shard:
        parallelism = (f"row-shard x{world}: " + (
            "outputs written to every rank over NVLink (CUDA IPC peer stores of flagged words) inside "
            "the kernel" if persistent else "NCCL all-gather after every GEMV") if world > 1
            else "single GPU (one shard)")
    else:
        parallelism = (f"{world} replicas: one full chain per GPU on its own inputs, no collective in "
                       "the data path" if world > 1 else "single GPU")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong" if shard else "weak",
        "vs_baseline": None,
        "dtype": "int8 dp4a / fp32", "data": "synthetic",
        "config": {"workload": f"{args.workload} per-token GEMV chain",
                   "gemvs_per_step": len(spec.gemvs), "ncols": args.ncols,
                   "launch_table": smithy or "built-in launch shapes",
                   "groups_per_step": n_groups if persistent else None,
                   "quantizations_per_step": n_groups if persistent else n_quantize,
                   "bytes_per_step": total_bytes, "weight_bytes": spec.weight_bytes(),
                   "us_per_token": round(ms * 1e3, 1), "pct_of_hbm_peak": round(100 * value / hbm_peak, 1),
                   "pct_of_8TBps": round(100 * value / 8000.0, 1),
                   "l2": "inputs larger than L2 (weights stream from HBM every step)",
                   "parallelism": parallelism,
                   "executor": ("one persistent cooperative kernel per token: groups of GEMVs sharing an "
                                "input, Q8_1 quantisation in-kernel, "
                                + ("each group reading its producer's output as it arrives (flagged words)"
                                   if dataflow else "fixed inputs")
                                if persistent else
                                "CUDA graph of quantize + MMVQ launches on fixed inputs, programmatic "
                                "dependent launch"),
                   "gate_up": "one gate/up GEMV per pair, silu(gate) * up" if persistent or args.glu
                              else "grouped gate and up GEMVs",
                   **({"persistent": pinfo} if persistent else
                      {"coresident_kernels_per_sm": args.coresident, "grouped_launches": bool(args.grouped)})},
        "e2e": e2e, "roofline": roofline, "gpu_launches": launches_per_step * args.steps,
        "device_status": status,
    }
    if trace is not None:
        line["trace"] = trace
    if extras:
        line["extras"] = extras
    if clk is not None:
        line["clocks"] = clk
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, args.cpu_seconds)
        try:
            line["cpu_baseline"]["reference_dependency"] = reference_dependency(args.workload)
        except ImportError as e:  # gguf-py missing on the host
            line["cpu_baseline"]["reference_dependency"] = {"unavailable": str(e)}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_anvil(args)


if __name__ == "__main__":
    main()
