"""kernel-anvil command line (B200 build).

Same sub-command names, arguments and defaults as the reference's kernel_anvil/cli.py:1101-1238
where the command belongs to the MMVQ path; every timing runs the real sm_100a kernels:

  gguf-optimize MODEL.gguf [--draft D.gguf]... [--no-bench] [--legacy-keys]
      tune every unique GEMV shape (nwarps x rows_per_block grid, each candidate checked
      against the stock launch's output) and write ~/.cache/smithy/<stem>.json (cli.py:412-581)
  merge-configs A.json B.json -o OUT.json      first input wins shared cells (cli.py:584-623)
  sweep RUNNER.py / profile RUNNER.py          runner-script convention (cli.py:58-230)
  autoforge MODEL.gguf | --chain NAME          full grid sweep per shape (autoforge.py:232-420)
  chain-sweep --chain NAME [--nwarps 1,2,4,8]  one global nwarps chosen by whole-token chain
                                               time (the llama-sweep idea, llama_sweep.py:229-342)
  bench-gemv --quant Q4_K --n 4096 --k 4096    one shape, buffers rotated past L2, JSON out
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile
import time
from pathlib import Path

from rich.console import Console
from rich.table import Table

console = Console()


# ---------------------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------------------

def _atomic_write_text(path: Path, text: str) -> None:
    """Write through a temp file in the same directory + rename, so a failed write leaves
    neither a truncated target nor a stray temp file (cli.py:548-560 of the reference)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=str(path.parent), suffix=".json.tmp")
    try:
        with os.fdopen(fd, "w") as f:
            f.write(text)
        os.replace(tmp, str(path))
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def _int_list(text: str) -> list[int]:
    vals = [int(x) for x in text.split(",") if x.strip()]
    if not vals or any(v <= 0 for v in vals):
        raise ValueError("All values must be positive")
    return vals


def _format_config(cfg: dict) -> str:
    return " ".join(f"{k}={cfg[k]}" for k in sorted(cfg))


def _load_runner(path: str):
    """Import a runner script: setup() -> inputs, run(inputs, **config) -> output,
    reference(inputs) -> expected output; optional DATA_BYTES, BASELINE_CONFIG, PARAM_SPACE."""
    p = Path(path).resolve()
    if not p.exists():
        console.print(f"[red]Runner not found: {p}[/red]")
        sys.exit(1)
    spec = importlib.util.spec_from_file_location("runner", p)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    for fn in ("setup", "run", "reference"):
        if not hasattr(mod, fn):
            console.print(f"[red]Runner {p.name} has no {fn}()[/red]")
            sys.exit(1)
    return mod


def _gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def heuristic_config(quant: str, n: int, k: int) -> dict:
    """The library's built-in B200 launch for a shape (default_config in csrc/anvil_abi.cu),
    used by --no-bench where the reference fell back to its RDNA3 heuristic (cli.py:273-336)."""
    if n < 2048:
        return {"nwarps": 8, "rows_per_block": 1}
    return {"nwarps": 4, "rows_per_block": 2 if k >= 8192 else 4}


# ---------------------------------------------------------------------------------------
# gguf-optimize
# ---------------------------------------------------------------------------------------

def _tune_shape_cli(quant: str, n: int, k: int, max_configs: int, warmup: int, runs: int):
    """Time up to max_configs launches of one (quant, N, K), stock launch first.  Returns
    (winning config, stock latency in us, stock / winner).  Only candidates whose output
    matches the stock launch's are eligible."""
    from kernel_anvil.autoforge import sweep_shape

    res = sweep_shape(quant, n, k, warmup=max(warmup, 1), runs=max(runs, 20))
    res = res[:max(1, max_configs)]
    stock = res[0]
    good = [r for r in res if r.correct] or [stock]
    best = min(good, key=lambda r: r.latency_us)
    speedup = stock.latency_us / best.latency_us if best.latency_us > 0 else None
    return {"nwarps": best.nwarps, "rows_per_block": best.rows_per_block}, stock.latency_us, speedup


def _profile_gguf_shapes(profile, *, no_bench: bool, args, label: str, codegen_configs: dict,
                         results_table: list, speedups: dict, legacy_keys: bool,
                         tune=None) -> None:
    """Tune every unique shape of one model into the shared dicts.  A shape an earlier model
    of the same run already tuned is reused; a failed shape stays absent so a later model
    can retry it (the reference's _profile_gguf_shapes, cli.py:338-409)."""
    from kernel_anvil.quants import get_quant_info

    tune = tune or _tune_shape_cli
    shapes = profile.unique_shapes if legacy_keys else profile.gemv_shapes()
    prefix = f"[{label}] " if label else ""
    verb = "Generating heuristic configs for" if no_bench else "Tuning"
    console.print(f"[bold]{prefix}{verb} {len(shapes)} unique GEMV workloads...[/bold]\n")
    for i, ((qt, a, b), count) in enumerate(sorted(shapes.items()), 1):
        n, k = (b, a) if legacy_keys else (a, b)  # legacy keys are (ne0, ne1) = (cols, rows)
        key = (qt, a, b)
        tag = f"  {prefix}[{i}/{len(shapes)}] {qt} ({a}, {b}) x{count}"
        if key in codegen_configs:
            console.print(f"{tag}: [dim]reused[/dim]")
            continue
        info = get_quant_info(qt)
        if info is None or k % info.qk:
            console.print(f"{tag}: [dim]skipped (no MMVQ kernel for this type)[/dim]")
            continue
        if no_bench:
            cfg = heuristic_config(info.name, n, k)
            codegen_configs[key] = cfg
            console.print(f"{tag}: nwarps={cfg['nwarps']} rows={cfg['rows_per_block']} (heuristic)")
            results_table.append((label, qt, a, b, count, cfg, 0.0, None, 0.0))
            continue
        t0 = time.monotonic()
        try:
            cfg, base_us, speedup = tune(info.name, n, k, args.max_configs, args.warmup, args.runs)
        except Exception as e:  # leave the slot absent: a later model may retry it
            console.print(f"{tag}: [red]FAILED: {e}[/red]")
            results_table.append((label, qt, a, b, count, None, 0.0, None, time.monotonic() - t0))
            continue
        dt = time.monotonic() - t0
        sp = f"{speedup:.2f}x" if speedup is not None else "-"
        console.print(f"{tag}: nwarps={cfg['nwarps']} rows={cfg['rows_per_block']} ({sp}, {dt:.1f}s)")
        codegen_configs[key] = cfg
        if speedup is not None:
            speedups[key] = float(speedup)
        results_table.append((label, qt, a, b, count, cfg, base_us, speedup, dt))


def cmd_gguf_optimize(args, tune=None) -> None:
    from kernel_anvil.codegen import generate_config_header, generate_runtime_config
    from kernel_anvil.gguf import parse_gguf, print_model_summary
    from kernel_anvil.specs import B200, detect_gpu

    gguf_path = Path(args.gguf)
    if not gguf_path.exists():
        console.print(f"[red]GGUF file not found: {gguf_path}[/red]")
        sys.exit(1)
    draft_paths = []
    for raw in args.draft or []:
        dp = Path(raw)
        if not dp.exists():
            console.print(f"[red]Draft GGUF not found: {dp}[/red]")
            sys.exit(1)
        draft_paths.append(dp)

    no_bench = args.no_bench
    if not no_bench and tune is None and not _gpu_available():
        console.print("[yellow]No CUDA GPU visible. Falling back to --no-bench mode.[/yellow]")
        no_bench = True
    gpu_spec = (detect_gpu() or B200) if not no_bench else B200

    console.print(f"\n[bold]Parsing {gguf_path.name}...[/bold]")
    target = parse_gguf(gguf_path)
    print_model_summary(target)
    drafts = []
    for dp in draft_paths:
        console.print(f"\n[bold]Parsing draft {dp.name}...[/bold]")
        prof = parse_gguf(dp)
        print_model_summary(prof)
        drafts.append((dp, prof))
    if not target.unique_shapes and not any(p.unique_shapes for _, p in drafts):
        console.print("[yellow]No 2D weight tensors found in any model.[/yellow]")
        sys.exit(0)

    configs: dict = {}
    speedups: dict = {}
    rows: list = []
    t0 = time.monotonic()
    _profile_gguf_shapes(target, no_bench=no_bench, args=args, label="target" if drafts else "",
                         codegen_configs=configs, results_table=rows, speedups=speedups,
                         legacy_keys=args.legacy_keys, tune=tune)
    for idx, (_, prof) in enumerate(drafts, 1):
        _profile_gguf_shapes(prof, no_bench=no_bench, args=args,
                             label="draft" if len(drafts) == 1 else f"draft{idx}",
                             codegen_configs=configs, results_table=rows, speedups=speedups,
                             legacy_keys=args.legacy_keys, tune=tune)
    total = time.monotonic() - t0

    table = Table(title="Optimization Results")
    if drafts:
        table.add_column("Source", style="magenta")
    table.add_column("Quant", style="cyan")
    for col in ("N", "K", "Count", "nwarps", "rows", "Stock (us)", "Speedup", "Time"):
        table.add_column(col, justify="right")
    for label, qt, a, b, count, cfg, base_us, speedup, dt in rows:
        fail = "[red]FAIL[/red]"
        row = [qt, str(a), str(b), str(count),
               str(cfg["nwarps"]) if cfg else fail, str(cfg["rows_per_block"]) if cfg else fail,
               f"{base_us:.1f}" if base_us else "-",
               f"{speedup:.2f}x" if speedup is not None else "-", f"{dt:.1f}s"]
        if drafts:
            row.insert(0, label or "target")
        table.add_row(*row)
    console.print(table)
    console.print(f"\nTotal tuning time: {total:.1f}s")

    model_name = "+".join([target.name] + [p.name for _, p in drafts])
    text = generate_runtime_config(configs, gpu_name=gpu_spec.gfx, model_name=model_name,
                                   priorities=speedups if drafts else None)
    cache_path = Path.home() / ".cache" / "smithy" / f"{gguf_path.stem}.json"
    _atomic_write_text(cache_path, text)
    console.print(f"\n[bold green]Config cached to {cache_path}[/bold green]")
    if drafts:
        console.print(f"[dim]Run: SMITHY_CONFIG={cache_path} llama-server -m {args.gguf} "
                      f"-md {drafts[0][0]} -ngl 999[/dim]")
        if len(drafts) > 1:
            console.print("[dim]      (merged config also covers: "
                          f"{', '.join(str(dp) for dp, _ in drafts[1:])})[/dim]")
    else:
        console.print(f"[dim]Run: SMITHY_MODEL={args.gguf} llama-server -m {args.gguf} -ngl 999[/dim]")
    if args.output != "smithy-config.h":
        hdr = generate_config_header(configs, gpu_name=f"{gpu_spec.gfx} ({gpu_spec.name})",
                                     model_name=model_name)
        Path(args.output).write_text(hdr)
        console.print(f"[dim]C header also written to {args.output}[/dim]")


# ---------------------------------------------------------------------------------------
# merge-configs
# ---------------------------------------------------------------------------------------

def cmd_merge_configs(args) -> None:
    from kernel_anvil.codegen import merge_runtime_configs

    payloads = []
    for raw in args.inputs:
        p = Path(raw)
        if not p.exists():
            console.print(f"[red]Config not found: {p}[/red]")
            sys.exit(1)
        try:
            with open(p) as f:
                payloads.append(json.load(f))
        except (json.JSONDecodeError, UnicodeDecodeError) as e:
            console.print(f"[red]Invalid JSON in {p}: {e}[/red]")
            sys.exit(1)
    merged = merge_runtime_configs(payloads, gpu_name=args.gpu, model_name=args.model)
    out = Path(args.output)
    _atomic_write_text(out, json.dumps(merged, indent=2))
    cells = merged.get("configs") or {}
    console.print(f"[bold green]Merged {len(payloads)} configs -> {out}[/bold green]")
    console.print(f"[dim]{len(cells)} quant types, {sum(len(v) for v in cells.values())} cells[/dim]")


# ---------------------------------------------------------------------------------------
# runner-script sweep / profile
# ---------------------------------------------------------------------------------------

def cmd_sweep(args) -> None:
    from kernel_anvil.analyze import classify
    from kernel_anvil.profile import profile_kernel
    from kernel_anvil.specs import B200, detect_gpu
    from kernel_anvil.sweep import generate_configs
    from kernel_anvil.verify import verify_and_bench

    runner = _load_runner(args.runner)
    gpu = detect_gpu() or B200
    inputs = runner.setup()
    ref = runner.reference(inputs)
    base_cfg = dict(getattr(runner, "BASELINE_CONFIG", {}))
    data_bytes = getattr(runner, "DATA_BYTES", None)

    def fn(cfg):
        return runner.run(inputs, **cfg)

    console.print(f"\n[bold]Profiling baseline {_format_config(base_cfg) or '(no knobs)'}...[/bold]")
    report = classify(profile_kernel(fn, base_cfg, data_bytes, gpu, args.warmup, args.runs), gpu)
    base = verify_and_bench(fn, ref, base_cfg, args.warmup, args.runs, args.atol, args.rtol, data_bytes)
    console.print(f"Baseline latency: [cyan]{base.latency_us:.1f} us[/cyan]"
                  + ("" if base.correct else " [red](baseline output differs from reference)[/red]"))
    console.print(f"Bottleneck: [yellow]{report.classification}[/yellow] "
                  f"(severity {report.severity:.2f})")
    configs = generate_configs(report, base_cfg or None, args.max_configs,
                               param_space=getattr(runner, "PARAM_SPACE", None))
    if not configs:
        console.print("[yellow]No configs to sweep (launch_overhead: fuse instead)[/yellow]")
        return
    results = []
    for i, cfg in enumerate(configs, 1):
        try:
            results.append(verify_and_bench(fn, ref, cfg, args.warmup, args.runs, args.atol,
                                            args.rtol, data_bytes, base.latency_us))
        except Exception as e:
            console.print(f"  config {i}/{len(configs)} ({_format_config(cfg)}) failed: {e}")
    correct = sorted((r for r in results if r.correct), key=lambda r: r.latency_us)
    ranked = correct + [r for r in results if not r.correct]
    table = Table(title="Sweep Results")
    for col in ("#", "Config", "Latency (us)", "BW (GB/s)", "Speedup", "Status"):
        table.add_column(col)
    for i, r in enumerate(ranked, 1):
        table.add_row(str(i), _format_config(r.config), f"{r.latency_us:.1f}",
                      f"{r.bandwidth_gbs:.1f}" if r.bandwidth_gbs else "-",
                      f"{r.speedup:.2f}x" if r.speedup else "-",
                      "[green]OK[/green]" if r.correct else "[red]FAIL[/red]")
    console.print(table)
    if correct:
        console.print(f"\n[bold green]Winner:[/bold green] {_format_config(correct[0].config)}")
    else:
        console.print("\n[red]No correct configs found.[/red]")


def cmd_profile(args) -> None:
    from kernel_anvil.analyze import classify
    from kernel_anvil.profile import profile_kernel
    from kernel_anvil.specs import B200, detect_gpu

    import torch

    runner = _load_runner(args.runner)
    gpu = detect_gpu() or B200
    cfg = dict(getattr(runner, "BASELINE_CONFIG", {}))
    if args.ncu_csv and not torch.cuda.is_available():
        # a recorded capture classified without a GPU: time and DRAM bytes come from the
        # CSV; registers, shared memory and occupancy are unknown (0) without the device
        from kernel_anvil.analyze import ProfileMetrics

        console.print("[yellow]No GPU: classifying the recorded ncu capture alone[/yellow]")
        m = ProfileMetrics(duration_ns=0.0,
                           threads_per_block=cfg.get("nwarps", 0) * 32 or 128)
    else:
        inputs = runner.setup()
        m = profile_kernel(lambda c: runner.run(inputs, **c), cfg, getattr(runner, "DATA_BYTES", None),
                           gpu, args.warmup, args.runs)
    if args.ncu or args.ncu_csv:
        from kernel_anvil.profile import apply_ncu, parse_ncu_csv, profile_runner_ncu

        rows = (parse_ncu_csv(Path(args.ncu_csv).read_text()) if args.ncu_csv
                else profile_runner_ncu(args.runner, args.ncu_kernel))
        m = apply_ncu(m, rows)
    report = classify(m, gpu)
    table = Table(title="Profile Metrics")
    table.add_column("Metric", style="cyan")
    table.add_column("Value", justify="right")
    for k, v in (("Duration", f"{m.duration_ns:.0f} ns"), ("Registers/thread", str(m.regs_per_thread)),
                 ("Shared memory", f"{m.smem_bytes} bytes"),
                 ("Local memory (spills)", f"{m.spill_bytes} bytes"),
                 ("Bandwidth", f"{m.bandwidth_gbs:.1f} GB/s"),
                 ("DRAM bytes (ncu)", "-" if m.dram_bytes is None else str(m.dram_bytes)),
                 ("Occupancy", f"{m.occupancy_pct:.1f}%"), ("Limiting factor", m.limiting_factor)):
        table.add_row(k, v)
    console.print(table)
    console.print(f"\n[bold]Classification:[/bold] {report.classification} "
                  f"(severity {report.severity:.2f})")
    for d in report.directions:
        console.print(f"  - {d}")


# ---------------------------------------------------------------------------------------
# autoforge / chain-sweep / bench-gemv
# ---------------------------------------------------------------------------------------

def cmd_autoforge(args) -> None:
    from kernel_anvil.autoforge import autoforge

    try:
        nwarps, rpb = _int_list(args.nwarps), _int_list(args.rpb)
    except ValueError as e:
        console.print(f"[red]Invalid nwarps/rpb values: {e}[/red]")
        sys.exit(1)
    shapes, name = None, None
    if args.chain:
        from kernel_anvil.chains import get_chain

        shapes, name = get_chain(args.chain).unique_shapes(), args.chain
    elif not args.gguf:
        console.print("[red]autoforge needs a GGUF file or --chain NAME[/red]")
        sys.exit(1)
    elif not Path(args.gguf).exists():
        console.print(f"[red]GGUF file not found: {args.gguf}[/red]")
        sys.exit(1)
    console.print(f"Sweeping nwarps={nwarps} x rpb={rpb} = {len(nwarps) * len(rpb)} configs per shape")
    res = autoforge(model_path=args.gguf, shapes=shapes, model_name=name, nwarps_candidates=nwarps,
                    rpb_candidates=rpb, output=args.output, legacy_keys=args.legacy_keys,
                    ncols=args.ncols)
    console.print(f"Config written to {res.config_path} ({res.total_time_s:.1f} s)")
    if args.json:
        with open(args.json, "w") as f:
            json.dump([r.__dict__ for r in res.all_results], f, indent=1)


def chain_tensors(spec, layers: int) -> list[tuple[str, str, int, int]]:
    """(tensor name, quant, N rows, K cols) of a chain's GEMVs in its first `layers` decoder
    layers (blk.<i>.<name>.weight), its other GEMVs once per unique shape (name.weight)."""
    out, seen = [], set()
    for g in spec.gemvs:
        parts = g.name.split(".")
        if parts[0] == "blk" and len(parts) > 2 and parts[1].isdigit():
            if int(parts[1]) < layers:
                out.append((g.name + ".weight", g.qt, g.nrows, g.K))
        elif (g.qt, g.nrows, g.K) not in seen:
            seen.add((g.qt, g.nrows, g.K))
            out.append((g.name + ".weight", g.qt, g.nrows, g.K))
    return out


def cmd_write_gguf(args) -> None:
    from kernel_anvil.chains import CHAINS, get_chain
    from kernel_anvil.gguf import write_gguf

    if args.chain not in CHAINS:
        console.print(f"[red]Unknown chain {args.chain!r} (known: {', '.join(CHAINS)})[/red]")
        sys.exit(1)
    if args.layers < 1:
        console.print("[red]--layers must be at least 1[/red]")
        sys.exit(1)
    tensors = chain_tensors(get_chain(args.chain), args.layers)
    path = write_gguf(args.output, tensors, name=args.chain, arch=args.chain.split("_")[0],
                      seed=args.seed)
    console.print(f"Wrote {path}: {len(tensors)} tensors")


def cmd_chain_sweep(args) -> None:
    """Time a whole decode chain (CUDA graph, PDL) once with the built-in per-shape launch and
    once per global nwarps; report us/token and optionally write the winner as smithy JSON."""
    import torch

    from kernel_anvil.autoforge import configs_json
    from kernel_anvil.chains import DeviceChain, get_chain

    try:
        candidates = _int_list(args.nwarps)
    except ValueError as e:
        console.print(f"[red]Invalid nwarps values: {e}[/red]")
        sys.exit(1)
    spec = get_chain(args.chain)
    results = []
    for nw in [0] + candidates:
        dc = DeviceChain(spec, nwarps=nw)
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            dc.instantiate(pdl=True)
            for _ in range(max(args.warmup, 1)):
                dc.launch()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.runs):
                dc.launch()
            e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000 / args.runs
        results.append((nw, us))
        console.print(f"  nwarps={'built-in' if nw == 0 else nw}: {us:.1f} us/token "
                      f"({dc.algorithmic_bytes / us / 1e3:.0f} GB/s)")
        dc.close()
        del dc
        torch.cuda.empty_cache()
    best_nw, best_us = min(results, key=lambda r: r[1])
    console.print(f"[bold green]Best: nwarps={'built-in' if best_nw == 0 else best_nw} "
                  f"{best_us:.1f} us/token ({results[0][1] / best_us:.2f}x vs built-in)[/bold green]")
    if args.output and best_nw:
        from types import SimpleNamespace

        winners = {s: SimpleNamespace(nwarps=best_nw,
                                      rows_per_block=heuristic_config(*s)["rows_per_block"])
                   for s in spec.unique_shapes()}
        _atomic_write_text(Path(args.output), configs_json(winners, "sm_100a", args.chain))
        console.print(f"Config written to {args.output}")


def cmd_bench_gemv(args) -> None:
    from kernel_anvil import mmvq as ops
    from kernel_anvil.verify import bench_gemv

    if args.tensor_cores == "off":
        ops.set_tensor_core_min_cols(0)
    for n in _int_list(args.n):
        for k in _int_list(args.k):
            for pdl in ([False, True] if args.pdl == "both" else [args.pdl == "on"]):
                res = bench_gemv(args.quant, n, k, ncols=args.ncols, nwarps=args.nwarps,
                                 rows_per_block=args.rpb, warmup=args.warmup, runs=args.runs,
                                 rotate_bytes=int(args.rotate_mb * 1e6), pdl=pdl)
                res["tensor_cores"] = args.tensor_cores
                print(json.dumps(res), flush=True)


# ---------------------------------------------------------------------------------------

def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="kernel-anvil",
                                     description="Shape-tuned MMVQ kernels for NVIDIA B200 (sm_100a)")
    sub = parser.add_subparsers(dest="command")

    p = sub.add_parser("sweep", help="End-to-end optimization sweep of a runner script")
    p.add_argument("runner", help="Path to runner script")
    p.add_argument("--max-configs", type=int, default=20, help="Max configs to try (default: 20)")
    p.add_argument("--warmup", type=int, default=5, help="Warmup iterations (default: 5)")
    p.add_argument("--runs", type=int, default=10, help="Timed iterations (default: 10)")
    p.add_argument("--atol", type=float, default=1e-2, help="Absolute tolerance (default: 1e-2)")
    p.add_argument("--rtol", type=float, default=1e-2, help="Relative tolerance (default: 1e-2)")
    p.set_defaults(fn=cmd_sweep)

    p = sub.add_parser("profile", help="Profile a runner script's kernel and classify its bottleneck")
    p.add_argument("runner", help="Path to runner script")
    p.add_argument("--warmup", type=int, default=5, help="Warmup iterations (default: 5)")
    p.add_argument("--runs", type=int, default=20, help="Timed iterations (default: 20)")
    p.add_argument("--ncu", action="store_true",
                   help="also read DRAM bytes and device time from ncu (one pass, clocks left alone)")
    p.add_argument("--ncu-kernel", default="mmvq", help="ncu kernel name regex (default: mmvq)")
    p.add_argument("--ncu-csv", default=None,
                   help="use a recorded `ncu --csv` metrics log instead of running ncu")
    p.set_defaults(fn=cmd_profile)

    p = sub.add_parser("gguf-optimize", help="Parse GGUF, tune shapes on the real kernels, write smithy JSON")
    p.add_argument("gguf", help="Path to GGUF model file")
    p.add_argument("--output", default="smithy-config.h",
                   help="C header path, written when not the default (default: smithy-config.h)")
    p.add_argument("--max-configs", type=int, default=15, help="Max configs per shape (default: 15)")
    p.add_argument("--warmup", type=int, default=3, help="Warmup iterations (default: 3)")
    p.add_argument("--runs", type=int, default=5, help="Timed iterations (default: 5)")
    p.add_argument("--no-bench", action="store_true",
                   help="Skip GPU benchmarking, use the built-in B200 launch (works without GPU)")
    p.add_argument("--draft", action="append", metavar="GGUF",
                   help="Draft model GGUF (speculative decoding); may be repeated. Tuned together "
                        "with the target into one config keyed under the target stem.")
    p.add_argument("--legacy-keys", action="store_true",
                   help="key cells by (ne0, ne1) as the reference does, instead of (rows, cols)")
    p.set_defaults(fn=cmd_gguf_optimize)

    p = sub.add_parser("merge-configs", help="Merge several kernel-anvil JSON configs into one")
    p.add_argument("inputs", nargs="+", help="Input config JSON files (priority = argument order)")
    p.add_argument("-o", "--output", required=True, help="Output merged config path")
    p.add_argument("--gpu", help="Override gpu field in merged output")
    p.add_argument("--model", help="Override model field in merged output")
    p.set_defaults(fn=cmd_merge_configs)

    p = sub.add_parser("autoforge", help="Sweep the real MMVQ kernels per shape and write smithy JSON")
    p.add_argument("gguf", nargs="?", help="GGUF model file (or use --chain)")
    p.add_argument("--chain", help="built-in decode chain instead of a GGUF (qwen3_8b, llama3_70b, ...)")
    p.add_argument("--nwarps", default="1,2,4,8", help="nwarps to sweep (default: 1,2,4,8)")
    p.add_argument("--rpb", default="1,2,4", help="rows_per_block to sweep (default: 1,2,4)")
    p.add_argument("--ncols", type=int, default=1)
    p.add_argument("--output", help="config path (default ~/.cache/smithy/<model>.json)")
    p.add_argument("--legacy-keys", action="store_true",
                   help="key cells by the reference's (ne0, ne1) instead of (rows, cols)")
    p.add_argument("--json", help="also write every measured point here")
    p.set_defaults(fn=cmd_autoforge)

    p = sub.add_parser("write-gguf", help="Write a GGUF of a built-in chain's weight tensors "
                                          "(seeded synthetic blocks) for gguf-optimize / autoforge")
    p.add_argument("chain", help="built-in chain (qwen3_8b, qwen3_0_6b, llama3_70b, qwen35_27b)")
    p.add_argument("output", help="GGUF path to write")
    p.add_argument("--layers", type=int, default=1,
                   help="decoder layers to write (the tail, e.g. the output head, is always written); "
                        "every unique GEMV shape appears from one layer on (default: 1)")
    p.add_argument("--seed", type=int, default=0)
    p.set_defaults(fn=cmd_write_gguf)

    p = sub.add_parser("chain-sweep", help="Pick one nwarps for a whole decode chain by chain time")
    p.add_argument("--chain", default="qwen3_8b")
    p.add_argument("--nwarps", default="1,2,4,8", help="Comma-separated nwarps to try (default: 1,2,4,8)")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--runs", type=int, default=10)
    p.add_argument("--output", help="write the winner as smithy JSON here")
    p.set_defaults(fn=cmd_chain_sweep)

    p = sub.add_parser("bench-gemv", help="Time one quantized GEMV shape (L2-defeating buffer rotation)")
    p.add_argument("--quant", default="Q4_K")
    p.add_argument("--n", default="4096", help="rows (output features); comma list allowed")
    p.add_argument("--k", default="4096", help="columns (input features); comma list allowed")
    p.add_argument("--ncols", type=int, default=1)
    p.add_argument("--nwarps", type=int, default=0)
    p.add_argument("--rpb", type=int, default=0)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--runs", type=int, default=100)
    p.add_argument("--rotate-mb", type=float, default=512.0,
                   help="distinct weight copies cycled through (> L2 so each launch reads HBM)")
    p.add_argument("--pdl", choices=["off", "on", "both"], default="off",
                   help="launch with programmatic dependent launch (consecutive launches overlap)")
    p.add_argument("--tensor-cores", choices=["on", "off"], default="on",
                   help="Q4_K / Q5_K with 2-8 columns: the mma.sync kernel (on) or the dp4a "
                        "kernels (off)")
    p.set_defaults(fn=cmd_bench_gemv)
    return parser


def main(argv=None) -> None:
    parser = build_parser()
    args = parser.parse_args(argv)
    if args.command is None:
        parser.print_help()
        sys.exit(1)
    args.fn(args)


if __name__ == "__main__":
    main()
