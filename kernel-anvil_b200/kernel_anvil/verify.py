"""Timing and verification of kernels on the GPU.

B200 replacement of the reference's kernel_anvil/verify.py:20-148: latency is measured with
CUDA events on the launching stream, bandwidth is algorithmic bytes over latency, and a
result is "correct" when it matches the reference output under allclose.  Single-GEMV
timing cycles through distinct weight copies (more bytes than L2 holds) inside a CUDA graph,
so every launch streams its weights from HBM and host launch cost is out of the picture.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass
from pathlib import Path

import torch

HAS_CUDA = torch.cuda.is_available()
L2_BYTES = 126 * 1024 * 1024  # B200


@dataclass
class VerifyResult:
    config: dict
    correct: bool
    max_diff: float          # max absolute difference from the reference output
    latency_us: float        # median latency in microseconds
    bandwidth_gbs: float | None
    speedup: float | None


def hbm_peak_gbs() -> float:
    """Measured HBM copy bandwidth of this pool (MEASURED_PEAKS.json), else 6650 GB/s."""
    for p in (Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json",):
        try:
            return float(json.loads(p.read_text())["hbm_gbs"])
        except Exception:
            pass
    return 6650.0


def _benchmark(fn, config: dict, warmup: int, runs: int) -> float:
    """Median latency (us) of fn(config) over `runs` launches, CUDA events per launch."""
    if not HAS_CUDA:
        raise RuntimeError("timing needs a CUDA device")
    torch.cuda.synchronize()
    for _ in range(warmup):
        fn(config)
    times = []
    stream = torch.cuda.current_stream()
    for _ in range(runs):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn(config)
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e) * 1000.0)
    return sorted(times)[len(times) // 2]


def verify_and_bench(kernel_fn, reference_output, config: dict, warmup: int = 5, runs: int = 10,
                     atol: float = 1e-2, rtol: float = 1e-2, data_bytes: int | None = None,
                     baseline_latency_us: float | None = None) -> VerifyResult:
    """Run kernel_fn(config), check it against reference_output, then time it."""
    out = kernel_fn(config)
    ref = reference_output
    correct = bool(torch.allclose(out.float(), ref.float(), atol=atol, rtol=rtol))
    max_diff = float((out.float() - ref.float()).abs().max().item())
    lat = _benchmark(kernel_fn, config, warmup, runs)
    bw = data_bytes / (lat * 1e-6) / 1e9 if data_bytes and lat > 0 else None
    sp = baseline_latency_us / lat if baseline_latency_us and lat > 0 else None
    return VerifyResult(config, correct, max_diff, lat, bw, sp)


class GemvBench:
    """One GEMV shape on `copies` distinct weight buffers, recorded as a CUDA graph that
    launches each copy once; replaying it times back-to-back launches from HBM."""

    def __init__(self, qt, n: int, k: int, ncols: int = 1, rotate_bytes: int = 512_000_000,
                 seed: int = 0, pdl: bool = False):
        from kernel_anvil import mmvq as ops
        from kernel_anvil.quants import gemv_bytes, make_weights_device, resolve_type

        self.info = resolve_type(qt)
        self.n, self.k, self.ncols, self.pdl = n, k, ncols, pdl
        wbytes = n * self.info.row_bytes(k)
        self.copies = max(2, math.ceil(max(rotate_bytes, 2 * L2_BYTES) / wbytes))
        w0 = make_weights_device(self.info, n, k, seed=seed)
        self.W = [w0] + [w0.clone() for _ in range(self.copies - 1)]
        g = torch.Generator(device="cuda")
        g.manual_seed(seed + 1)
        self.x = torch.randn((ncols, k), generator=g, device="cuda")
        self.xq = ops.quantize_q8_1(self.x)
        self.y = torch.empty((ncols, n), device="cuda")
        self.bytes = gemv_bytes(self.info, n, k, ncols)
        self.stream = torch.cuda.Stream()
        self.graphs: dict = {}

    def run(self, nwarps: int = 0, rows_per_block: int = 0, W=None) -> torch.Tensor:
        from kernel_anvil import mmvq as ops

        return ops.mmvq(self.W[0] if W is None else W, self.info, self.xq, ncols=self.ncols,
                        nwarps=nwarps, rows_per_block=rows_per_block, out=self.y, pdl=self.pdl)

    def time(self, nwarps: int = 0, rows_per_block: int = 0, warmup: int = 3, runs: int = 50) -> float:
        """Mean microseconds per launch."""
        key = (nwarps, rows_per_block)
        with torch.cuda.stream(self.stream):
            if key not in self.graphs:
                for W in self.W[:2]:
                    self.run(nwarps, rows_per_block, W)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=self.stream):
                    for W in self.W:
                        self.run(nwarps, rows_per_block, W)
                self.graphs[key] = graph
            graph = self.graphs[key]
            reps = max(1, math.ceil(runs / self.copies))
            for _ in range(max(1, math.ceil(warmup / self.copies))):
                graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            for _ in range(reps):
                graph.replay()
            e1.record(self.stream)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1000.0 / (reps * self.copies)

    def close(self) -> None:
        self.graphs.clear()
        self.W.clear()


def bench_gemv(qt, n: int, k: int, ncols: int = 1, nwarps: int = 0, rows_per_block: int = 0,
               warmup: int = 10, runs: int = 100, rotate_bytes: int = 512_000_000,
               pdl: bool = False) -> dict:
    """Time one GEMV shape; returns latency, GB/s and % of the measured HBM peak."""
    from kernel_anvil import mmvq as ops

    b = GemvBench(qt, n, k, ncols, rotate_bytes, pdl=pdl)
    us = b.time(nwarps, rows_per_block, warmup, runs)
    plan = ops.plan(b.info, n, k, ncols, nwarps, rows_per_block)
    gbs = b.bytes / (us * 1e-6) / 1e9
    peak = hbm_peak_gbs()
    res = {"quant": b.info.name, "n": n, "k": k, "ncols": ncols, **plan, "us": round(us, 3),
           "bytes": b.bytes, "gbs": round(gbs, 1), "pct_of_hbm_peak": round(100 * gbs / peak, 1),
           "pct_of_8TBps": round(100 * gbs / 8000, 1), "copies": b.copies, "pdl": pdl}
    b.close()
    return res
