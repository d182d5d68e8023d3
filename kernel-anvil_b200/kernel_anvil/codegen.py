"""smithy config tables: bucketing, runtime JSON, merge, and the legacy C header.

Same interface and byte-identical output as the reference's kernel_anvil/codegen.py, so
configs written by either tool load into either loader:

* ``bucket_index`` -- buckets <=128, <=1024, <=4096, <=16384, larger (codegen.py:17-18,44-56;
  the C loader's smithy_get_bucket, patches/smithy-config.h:44-50).
* ``build_config_tables`` -- per quant type a 5x5 [n_bucket][k_bucket] table filled with
  DEFAULT_CONFIG; later entries win a shared cell unless ``priorities`` is given, in which
  case the higher priority wins and NaN / missing priorities count as -inf
  (codegen.py:68-130).
* ``generate_runtime_config`` -- ``{"gpu", "model", "configs": {"<ggml type id>":
  {"<nb>,<kb>": {"nwarps", "rows_per_block"}}}}`` with cells equal to DEFAULT_CONFIG left
  out (codegen.py:133-183).
* ``merge_runtime_configs`` -- first payload wins a cell; malformed parts are skipped
  (codegen.py:186-260).
* ``generate_config_header`` -- the compile-time table header (codegen.py:263-362).

The (n, k) of a key is whatever the caller passes; gguf-optimize passes true rows and
columns (see kernel_anvil.gguf for the reference's (ne0, ne1) convention).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass
from datetime import datetime, timezone

BUCKET_BOUNDARIES = (128, 1024, 4096, 16384)
NUM_BUCKETS = len(BUCKET_BOUNDARIES) + 1

# ggml_type enum values (ggml.h) indexing smithy_configs[GGML_TYPE_COUNT][5][5].
GGML_TYPE_MAP = {
    "F32": 0, "F16": 1,
    "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q8_1": 9,
    "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q8_K": 15,
    "IQ2_XXS": 16, "IQ2_XS": 17, "IQ3_XXS": 18, "IQ1_S": 19, "IQ4_NL": 20,
    # IQ1_M is ggml type 29 (gguf-py GGMLQuantizationType); the reference's map says 24,
    # ggml's I8, under which a tuned IQ1_M cell would never be looked up
    "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "IQ1_M": 29,
    "BF16": 30,
    "MXFP4": 39, "NVFP4": 40,
}
GGML_TYPE_COUNT = 41


@dataclass(frozen=True)
class ShapeConfig:
    """Launch config of one (quant, N, K) workload."""
    nwarps: int
    rows_per_block: int


DEFAULT_CONFIG = ShapeConfig(nwarps=4, rows_per_block=1)


def bucket_index(value: int) -> int:
    """Index of the first bucket whose boundary is >= value (4 when above all)."""
    for i, boundary in enumerate(BUCKET_BOUNDARIES):
        if value <= boundary:
            return i
    return len(BUCKET_BOUNDARIES)


def _priority(p) -> float:
    if p is None:
        return float("-inf")
    v = float(p)
    return float("-inf") if math.isnan(v) else v


def build_config_tables(
    configs: dict[tuple[str, int, int], dict],
    priorities: dict[tuple[str, int, int], float] | None = None,
) -> dict[str, list[list[ShapeConfig]]]:
    """{quant: [n_bucket][k_bucket] ShapeConfig} for every quant present in ``configs``."""
    tables: dict[str, list[list[ShapeConfig]]] = {}
    for qt in sorted({q for q, _, _ in configs}):
        table = [[DEFAULT_CONFIG] * NUM_BUCKETS for _ in range(NUM_BUCKETS)]
        best: dict[tuple[int, int], float] = {}
        for (q, n, k), cfg in configs.items():
            if q != qt:
                continue
            cell = (bucket_index(n), bucket_index(k))
            if priorities is not None:
                p = _priority(priorities.get((q, n, k)))
                if cell in best and p <= best[cell]:
                    continue
                best[cell] = p
            table[cell[0]][cell[1]] = ShapeConfig(cfg["nwarps"], cfg["rows_per_block"])
        tables[qt] = table
    return tables


def generate_runtime_config(
    configs: dict[tuple[str, int, int], dict],
    gpu_name: str = "gfx1100",
    model_name: str = "unknown",
    priorities: dict[tuple[str, int, int], float] | None = None,
) -> str:
    """Runtime JSON for the smithy loader (libanvil's anvil_smithy_* or smithy-config.h)."""
    out: dict = {"gpu": gpu_name, "model": model_name, "configs": {}}
    for qt, table in build_config_tables(configs, priorities=priorities).items():
        type_idx = GGML_TYPE_MAP.get(qt)
        if type_idx is None:
            continue
        cells = {
            f"{ni},{ki}": {"nwarps": table[ni][ki].nwarps, "rows_per_block": table[ni][ki].rows_per_block}
            for ni in range(NUM_BUCKETS)
            for ki in range(NUM_BUCKETS)
            if table[ni][ki] != DEFAULT_CONFIG
        }
        if cells:
            out["configs"][str(type_idx)] = cells
    return json.dumps(out, indent=2)


def merge_runtime_configs(
    payloads: list[dict],
    gpu_name: str | None = None,
    model_name: str | None = None,
) -> dict:
    """Merge parsed runtime configs; earlier payloads win shared cells.

    Non-dict payloads, ``configs`` sections, per-type maps and cells are skipped, so a
    partly malformed file degrades to fewer cells instead of an exception.
    """
    if not payloads:
        return {"gpu": gpu_name or "unknown", "model": model_name or "merged", "configs": {}}
    merged: dict[str, dict[str, dict]] = {}
    valid = [p for p in payloads if isinstance(p, dict)]
    for payload in valid:
        cfgs = payload.get("configs") or {}
        if not isinstance(cfgs, dict):
            continue
        for type_idx, cells in cfgs.items():
            if not isinstance(cells, dict):
                continue
            dst = merged.setdefault(str(type_idx), {})
            for key, cell in cells.items():
                if key in dst or not isinstance(cell, dict):
                    continue
                dst[str(key)] = dict(cell)
    if gpu_name is None:
        g = valid[0].get("gpu") if valid else None
        gpu_name = g if isinstance(g, str) else "unknown"
    if model_name is None:
        names = [p.get("model") if isinstance(p.get("model"), str) else "unknown" for p in valid]
        model_name = "+".join(names) if names else "merged"
    return {"gpu": gpu_name, "model": model_name, "configs": merged}


def _type_name(type_idx: int) -> str | None:
    for name, idx in GGML_TYPE_MAP.items():
        if idx == type_idx:
            return name
    return None


def generate_config_header(
    configs: dict[tuple[str, int, int], dict],
    gpu_name: str = "gfx1100 (7900 XTX)",
    model_name: str = "unknown",
) -> str:
    """C header with a compile-time smithy_configs[GGML_TYPE_COUNT][5][5] table.

    Cells equal to DEFAULT_CONFIG are written as {0, 0} (no override)."""
    tables = build_config_tables(configs)
    stamp = datetime.now(timezone.utc).strftime("%Y-%m-%d %H:%M UTC")
    L = [
        f"// smithy-config.h - Generated by kernel-anvil for {gpu_name}",
        f"// Model: {model_name}",
        f"// Generated: {stamp}",
        "//",
        "// Bucket boundaries: " + ", ".join(str(b) for b in BUCKET_BOUNDARIES),
        f"// Buckets per axis: {NUM_BUCKETS}",
        "//",
        "// Drop this file into ggml/src/ggml-cuda/ to replace the default smithy-config.h",
        "// Rebuild llama.cpp to apply shape-specific kernel configs.",
        "#pragma once",
        "",
        "struct smithy_shape_config {",
        "    int nwarps;         // 0 = use default (no override)",
        "    int rows_per_block; // 0 = use default (no override)",
        "};",
        "",
        "enum smithy_bucket : int {",
    ]
    L += [f"    SMITHY_BUCKET_LE_{b:<5d} = {i}," for i, b in enumerate(BUCKET_BOUNDARIES)]
    L += [
        f"    SMITHY_BUCKET_GT_{BUCKET_BOUNDARIES[-1]:<5d} = {len(BUCKET_BOUNDARIES)},",
        f"    SMITHY_NUM_BUCKETS     = {NUM_BUCKETS},",
        "};",
        "",
        "static inline smithy_bucket smithy_get_bucket(int value) {",
    ]
    L += [f"    if (value <= {b}) return static_cast<smithy_bucket>({i});"
          for i, b in enumerate(BUCKET_BOUNDARIES)]
    L += [
        f"    return static_cast<smithy_bucket>({len(BUCKET_BOUNDARIES)});",
        "}",
        "",
        "// Indexed by [ggml_type][N_bucket][K_bucket]",
        "// Non-zero entries override llama.cpp defaults. Zero = no override.",
        "#ifndef SMITHY_CONFIG_TABLE",
        "#define SMITHY_CONFIG_TABLE",
        f"static const smithy_shape_config smithy_configs[{GGML_TYPE_COUNT}]"
        "[SMITHY_NUM_BUCKETS][SMITHY_NUM_BUCKETS] = {",
    ]
    for type_idx in range(GGML_TYPE_COUNT):
        name = _type_name(type_idx)
        if name and name in tables:
            L.append(f"    // [{type_idx}] = GGML_TYPE_{name}")
            L.append("    {")
            for ni in range(NUM_BUCKETS):
                cells = []
                for ki in range(NUM_BUCKETS):
                    c = tables[name][ni][ki]
                    nw, rpb = (0, 0) if c == DEFAULT_CONFIG else (c.nwarps, c.rows_per_block)
                    cells.append(f"{{{nw:2d},{rpb:2d}}}")
                L.append(f"        {{{', '.join(cells)}}},")
            L.append("    },")
        else:
            L.append(f"    {{{{}}}},  // [{type_idx}] unused")
    L += ["};", "#endif // SMITHY_CONFIG_TABLE", "", "// Profiled types:"]
    L += [f"//   GGML_TYPE_{qt} = {GGML_TYPE_MAP.get(qt, '?')}" for qt in sorted(tables)]
    L.append("")
    return "\n".join(L)
