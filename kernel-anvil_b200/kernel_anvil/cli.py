"""kernel-anvil command line (B200 build).

Subcommands (same names and defaults as the reference's kernel_anvil/cli.py:1101-1238
where they exist there):

  gguf-optimize MODEL.gguf [--draft D.gguf] [--no-bench] [--legacy-keys]
                      tune every unique GEMV shape with the real sm_100a kernels and write
                      ~/.cache/smithy/<stem>.json
  merge-configs A.json B.json -o OUT.json   first input wins shared cells
  sweep RUNNER.py / profile RUNNER.py       runner-script convention (setup/run/reference)
  autoforge MODEL.gguf [--nwarps 1,2,4,8] [--rpb 1,2,4]   grid sweep of the real kernels
  bench-gemv --quant Q4_K --n 4096 --k 4096 [--ncols 1] [--nwarps 0] [--rpb 0]
                      time one GEMV shape with buffers rotated past L2 (prints JSON)
"""
from __future__ import annotations

import argparse
import json
import sys


def cmd_bench_gemv(args) -> None:
    from kernel_anvil.verify import bench_gemv

    for n in _int_list(args.n):
        for k in _int_list(args.k):
            for pdl in ([False, True] if args.pdl == "both" else [args.pdl == "on"]):
                res = bench_gemv(args.quant, n, k, ncols=args.ncols, nwarps=args.nwarps,
                                 rows_per_block=args.rpb, warmup=args.warmup, runs=args.runs,
                                 rotate_bytes=int(args.rotate_mb * 1e6), pdl=pdl)
                print(json.dumps(res), flush=True)


def _int_list(text: str) -> list[int]:
    vals = [int(x) for x in text.split(",") if x.strip()]
    if not vals or any(v <= 0 for v in vals):
        raise ValueError("All values must be positive")
    return vals


def cmd_autoforge(args) -> None:
    from kernel_anvil.autoforge import autoforge

    try:
        nwarps, rpb = _int_list(args.nwarps), _int_list(args.rpb)
    except ValueError as e:
        print(f"Invalid nwarps/rpb values: {e}", file=sys.stderr)
        sys.exit(1)
    shapes, name = None, None
    if args.chain:
        from kernel_anvil.chains import get_chain

        shapes, name = get_chain(args.chain).unique_shapes(), args.chain
    elif not args.gguf:
        print("autoforge needs a GGUF file or --chain NAME", file=sys.stderr)
        sys.exit(1)
    print(f"Sweeping nwarps={nwarps} x rpb={rpb} = {len(nwarps) * len(rpb)} configs per shape")
    res = autoforge(model_path=args.gguf, shapes=shapes, model_name=name, nwarps_candidates=nwarps,
                    rpb_candidates=rpb, output=args.output, legacy_keys=args.legacy_keys,
                    ncols=args.ncols)
    print(f"Config written to {res.config_path} ({res.total_time_s:.1f} s)")
    if args.json:
        rows = [r.__dict__ for r in res.all_results]
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="kernel-anvil",
                                     description="Shape-tuned MMVQ kernels for NVIDIA B200 (sm_100a)")
    sub = parser.add_subparsers(dest="command")

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
    p.set_defaults(fn=cmd_bench_gemv)

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
