"""Kernel profiling for bottleneck analysis (B200 replacement of kernel_anvil/profile.py:37-91).

``profile_kernel`` times a callable with CUDA events and returns ProfileMetrics.  When the
config names an MMVQ launch (``quant``/``n``/``k`` keys, as the gguf-optimize runner passes),
registers, spills (local memory), shared memory and occupancy come from the compiled kernel
(cudaFuncGetAttributes) and the library's launch plan instead of the reference's estimates
(kernel_anvil/profile.py:7-34, the "Phase 2" real counters of :12-13).  ``ncu_metrics`` runs a
command under ncu for DRAM counters (the role rocprofv3 played for the reference,
kernel_anvil/llama_sweep.py:64-136); ``profile_runner_ncu`` does that for a runner script.
"""
from __future__ import annotations

import csv
import io
import shutil
import subprocess

from kernel_anvil.analyze import ProfileMetrics
from kernel_anvil.specs import GpuSpec
from kernel_anvil.verify import _benchmark


def _mmvq_resources(config: dict) -> tuple[int, int, int, int] | None:
    """(registers/thread, local bytes/thread, smem bytes, threads/block) of the MMVQ launch a
    config describes, from the compiled kernel and the launch plan."""
    try:
        from kernel_anvil import mmvq as ops

        args = (config["quant"], config["n"], config["k"], config.get("ncols", 1),
                config.get("nwarps", 0), config.get("rows_per_block", 0))
        plan = ops.plan(*args)
        attrs = ops.kernel_attributes(*args)
    except Exception:
        return None
    return attrs["regs_per_thread"], attrs["local_bytes"], plan["smem_bytes"], plan["nwarps"] * 32


def profile_kernel(kernel_fn, config: dict, data_bytes: int | None = None,
                   gpu_spec: GpuSpec | None = None, warmup: int = 5, runs: int = 20) -> ProfileMetrics:
    latency_us = _benchmark(kernel_fn, config, warmup, runs)
    bw = data_bytes / (latency_us * 1e-6) / 1e9 if data_bytes and latency_us > 0 else 0.0
    regs, spill, smem, threads = 0, 0, 0, config.get("nwarps", config.get("num_warps", 4)) * 32
    res = _mmvq_resources(config)
    if res is not None:
        regs, spill, smem, threads = res
    occ, factor = 0.0, "unknown"
    if gpu_spec is not None and (regs or smem):
        occ, factor = gpu_spec.occupancy(regs, smem, threads)
    return ProfileMetrics(duration_ns=latency_us * 1000, regs_per_thread=regs, smem_bytes=smem,
                          spill_bytes=spill, bandwidth_gbs=bw, occupancy_pct=occ, limiting_factor=factor,
                          threads_per_block=threads)


NCU_METRICS = ("gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum")


def parse_ncu_csv(text: str) -> list[dict]:
    """Rows of an `ncu --csv` metrics log as {kernel, metric: value} dicts (one per launch)."""
    lines = text.splitlines()
    start = next((i for i, ln in enumerate(lines) if ln.startswith('"ID"')), None)
    if start is None:
        return []
    reader = csv.reader(io.StringIO("\n".join(lines[start:])))
    hdr = next(reader)
    ki, mi, ui, vi, idi = (hdr.index(k) for k in ("Kernel Name", "Metric Name", "Metric Unit",
                                                   "Metric Value", "ID"))
    scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "nsecond": 1e-3, "ns": 1e-3,
             "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3}
    launches: dict[str, dict] = {}
    for r in reader:
        if len(r) <= vi:
            continue
        d = launches.setdefault(r[idi], {"kernel": r[ki].split("(")[0].replace("void ", "")})
        d[r[mi]] = float(r[vi].replace(",", "")) * scale.get(r[ui], 1.0)
    return list(launches.values())


def ncu_metrics(cmd: list[str], kernel_regex: str = "mmvq", launches: int = 1, skip: int = 0,
                metrics=NCU_METRICS, timeout: int = 600) -> list[dict]:
    """Run `cmd` under ncu (clocks left alone) and return per-launch metrics; times in µs."""
    ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
    full = [ncu, "--clock-control", "none", "--csv", "--metrics", ",".join(metrics),
            "-k", f"regex:{kernel_regex}", "-s", str(skip), "-c", str(launches), *cmd]
    r = subprocess.run(full, capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"ncu failed ({r.returncode}): {r.stderr[-2000:]}")
    return parse_ncu_csv(r.stdout)


def apply_ncu(metrics: ProfileMetrics, rows: list[dict]) -> ProfileMetrics:
    """metrics with ncu's DRAM bytes and device time per launch (means over the rows)."""
    if not rows:
        return metrics
    n = len(rows)
    dram = sum(r.get("dram__bytes_read.sum", 0.0) + r.get("dram__bytes_write.sum", 0.0) for r in rows) / n
    us = sum(r.get("gpu__time_duration.sum", 0.0) for r in rows) / n
    metrics.dram_bytes = int(dram)
    if us > 0:
        metrics.duration_ns = us * 1000.0
        metrics.bandwidth_gbs = dram / (us * 1e-6) / 1e9
    return metrics


def profile_runner_ncu(runner_path: str, kernel_regex: str = "mmvq", launches: int = 3,
                       timeout: int = 600) -> list[dict]:
    """ncu DRAM counters for a runner script's kernel: runs this module's runner mode
    (setup() once, run() with BASELINE_CONFIG `launches` times) under ncu, one pass of
    metrics, clocks left alone."""
    import sys

    cmd = [sys.executable, "-m", "kernel_anvil.profile", "--run-runner", str(runner_path),
           "--launches", str(launches)]
    return ncu_metrics(cmd, kernel_regex=kernel_regex, launches=launches, timeout=timeout)


def _run_runner_main(argv: list[str]) -> None:
    """Runner mode for ncu: load the script, setup(), run() with its BASELINE_CONFIG."""
    import argparse
    import importlib.util

    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--run-runner", required=True)
    ap.add_argument("--launches", type=int, default=3)
    a = ap.parse_args(argv)
    spec = importlib.util.spec_from_file_location("runner", a.run_runner)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    inputs = mod.setup()
    cfg = dict(getattr(mod, "BASELINE_CONFIG", {}))
    for _ in range(a.launches):
        mod.run(inputs, **cfg)
    torch.cuda.synchronize()


if __name__ == "__main__":
    import sys

    _run_runner_main(sys.argv[1:])
