"""autoforge: sweep the real sm_100a MMVQ kernel over launch configs per GEMV shape.

The reference's autoforge (kernel_anvil/autoforge.py:232-420) generates a HIP kernel per
(shape, nwarps, rows_per_block), compiles it with hipcc, times it on zero-filled buffers
without checking results, and writes the fastest per shape into smithy JSON.  Here the
kernels already exist (libanvil.so), so a sweep is: build one GemvBench per shape (seeded
quantized weights, buffers rotated past L2, CUDA-graph timing), run every grid point,
require its output to match the stock config's output, and keep the fastest correct one.

Grid: nwarps {1,2,4,8} x rows_per_block {1,2,4} (autoforge.py:254-257).  "Stock" is the
reference's llama.cpp baseline, nwarps=8 rows_per_block=1 (autoforge.py:338-347).
Output cells are written explicitly for every winner (as the reference autoforge does),
keyed by true (N rows, K cols) unless legacy_keys asks for the reference's (ne0, ne1).
"""
from __future__ import annotations

import json
import os
import tempfile
import time
from dataclasses import dataclass, field
from pathlib import Path

from kernel_anvil.codegen import GGML_TYPE_MAP, bucket_index

STOCK = {"nwarps": 8, "rows_per_block": 1}


@dataclass
class BenchResult:
    quant: str
    n: int
    k: int
    ncols: int
    nwarps: int
    rows_per_block: int
    latency_us: float
    bandwidth_gbs: float
    data_bytes: int
    correct: bool
    max_rel_diff: float = 0.0


@dataclass
class ForgeResult:
    model: str
    gpu_arch: str
    shapes: dict = field(default_factory=dict)   # (qt, n, k) -> winning BenchResult
    stock: dict = field(default_factory=dict)    # (qt, n, k) -> stock BenchResult
    all_results: list = field(default_factory=list)
    config_path: str | None = None
    total_time_s: float = 0.0

    def speedup(self, key) -> float | None:
        w, s = self.shapes.get(key), self.stock.get(key)
        if not w or not s or w.latency_us <= 0:
            return None
        return s.latency_us / w.latency_us


def sweep_shape(qt, n: int, k: int, ncols: int = 1, nwarps_candidates=(1, 2, 4, 8),
                rpb_candidates=(1, 2, 4), warmup: int = 3, runs: int = 40,
                rotate_bytes: int = 300_000_000, pdl: bool = False, tol: float = 1e-4) -> list[BenchResult]:
    """Time every (nwarps, rows_per_block) on one shape; results[0] is the stock config."""
    import torch

    from kernel_anvil.verify import GemvBench

    b = GemvBench(qt, n, k, ncols, rotate_bytes=rotate_bytes, pdl=pdl)
    try:
        ref = b.run(**STOCK).clone()
        scale = float(ref.abs().max().item()) or 1.0
        cands = [dict(STOCK)] + [{"nwarps": nw, "rows_per_block": r}
                                 for nw in nwarps_candidates for r in rpb_candidates
                                 if {"nwarps": nw, "rows_per_block": r} != STOCK]
        out = []
        for c in cands:
            y = b.run(**c)
            diff = float((y - ref).abs().max().item()) / scale
            us = b.time(c["nwarps"], c["rows_per_block"], warmup, runs)
            out.append(BenchResult(b.info.name, n, k, ncols, c["nwarps"], c["rows_per_block"], us,
                                   b.bytes / (us * 1e-6) / 1e9, b.bytes, diff <= tol, diff))
        torch.cuda.synchronize()
        return out
    finally:
        b.close()


def _atomic_write(path: Path, text: str) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=str(path.parent), suffix=".json.tmp")
    try:
        with os.fdopen(fd, "w") as f:
            f.write(text)
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def configs_json(winners: dict, gpu: str, model: str, legacy_keys: bool = False) -> str:
    """smithy JSON with one explicit cell per winner (later shapes win shared cells)."""
    out = {"gpu": gpu, "model": model, "configs": {}}
    for (qt, n, k), r in winners.items():
        tid = GGML_TYPE_MAP.get(qt)
        if tid is None:
            continue
        a, b = (k, n) if legacy_keys else (n, k)
        out["configs"].setdefault(str(tid), {})[f"{bucket_index(a)},{bucket_index(b)}"] = {
            "nwarps": r.nwarps, "rows_per_block": r.rows_per_block}
    return json.dumps(out, indent=2)


def autoforge(model_path: str | None = None, shapes: dict | None = None, model_name: str | None = None,
              nwarps_candidates=(1, 2, 4, 8), rpb_candidates=(1, 2, 4), output: str | None = None,
              legacy_keys: bool = False, ncols: int = 1, verbose: bool = True, **sweep_kw) -> ForgeResult:
    """Sweep every unique GEMV shape of a GGUF model (or of `shapes`: {(qt, N, K): count})
    and write the winners to ~/.cache/smithy/<model>.json (or `output`)."""
    from kernel_anvil.quants import get_quant_info
    from kernel_anvil.specs import B200

    t0 = time.monotonic()
    if shapes is None:
        if model_path is None:
            raise ValueError("need a GGUF path or a shape dict")
        from kernel_anvil.gguf import parse_gguf

        prof = parse_gguf(model_path)
        shapes = prof.gemv_shapes()
        model_name = model_name or Path(model_path).stem
    model_name = model_name or "shapes"
    res = ForgeResult(model=model_name, gpu_arch=B200.arch)
    for (qt, n, k), count in sorted(shapes.items()):
        info = get_quant_info(qt)
        if info is None or k % info.qk:
            if verbose:
                print(f"  {qt} ({n}, {k}) x{count}: SKIPPED (no MMVQ kernel for this type/shape)")
            continue
        rs = sweep_shape(info.name, n, k, ncols, nwarps_candidates, rpb_candidates, **sweep_kw)
        res.all_results += rs
        res.stock[(qt, n, k)] = rs[0]
        good = [r for r in rs if r.correct]
        if not good:
            if verbose:
                print(f"  {qt} ({n}, {k}) x{count}: FAILED (no candidate matched the stock output)")
            continue
        best = min(good, key=lambda r: r.latency_us)
        res.shapes[(qt, n, k)] = best
        if verbose:
            sp = res.speedup((qt, n, k))
            print(f"  {qt} ({n}, {k}) x{count}: nw={best.nwarps} rpb={best.rows_per_block} "
                  f"{best.latency_us:.2f}us {best.bandwidth_gbs:.0f}GB/s ({sp:.2f}x vs stock) "
                  f"[{len(rs)} tested]")
    path = Path(output) if output else Path.home() / ".cache" / "smithy" / f"{model_name}.json"
    _atomic_write(path, configs_json(res.shapes, res.gpu_arch, model_name, legacy_keys))
    res.config_path = str(path)
    res.total_time_s = time.monotonic() - t0
    return res
