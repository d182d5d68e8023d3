"""Regenerates the golden fixtures in tests/golden/ from the reference and its dependency.

Run in the build container (where the reference tree and gguf-py are present):

    python tests/golden/make_golden.py [--reference /root/reference] [--types IQ2_XXS ...]

Writes:
  dequant_<type>.npz   seeded GGUF-layout blocks and gguf-py ``gguf.quants.dequantize``
                       output (gguf 0.19.0, the reference's declared dependency).
  q8_0_gguf.npz        seeded activations and gguf-py's Q8_0 quantisation of them (the
                       closest pinned relative of Q8_1: same d = amax/127 rule).
  codegen.json         outputs of the reference's kernel_anvil.codegen (bucket_index,
                       generate_runtime_config, merge_runtime_configs,
                       generate_config_header) on fixed inputs, produced by importing the
                       reference package in a subprocess.
  smithy_loader.json   tables the reference's C++ loader (patches/smithy-config.h, built
                       by oracle/Makefile into oracle/_ref) reads from a battery of JSON
                       documents, malformed ones included.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "kernel-anvil_b200"))
sys.path.insert(0, str(REPO))

from kernel_anvil.quants import make_activation, make_weights  # noqa: E402

DEQUANT_CASES = {"Q4_K": (8, 512), "Q5_K": (8, 512), "Q6_K": (8, 512), "Q8_0": (8, 256),
                 "Q4_0": (8, 256), "Q4_1": (8, 256), "Q5_0": (8, 256), "Q5_1": (8, 256),
                 "Q2_K": (8, 512), "Q3_K": (8, 512), "IQ4_NL": (8, 256), "IQ4_XS": (8, 512),
                 "IQ2_XXS": (8, 512), "IQ2_XS": (8, 512), "IQ2_S": (8, 512), "IQ3_XXS": (8, 512),
                 "IQ3_S": (8, 512), "IQ1_S": (8, 512), "IQ1_M": (8, 512)}

# Inputs for the reference's codegen.  Keys are (quant, n, k) -> {nwarps, rows_per_block}.
CODEGEN_CASES = [
    {"name": "single", "configs": [["Q4_K", 4096, 4096, 8, 2]]},
    {"name": "default_cells_omitted", "configs": [["Q4_K", 4096, 4096, 4, 1], ["Q4_K", 12288, 4096, 8, 1]]},
    {"name": "multi_type", "configs": [["Q4_K", 4096, 4096, 4, 2], ["Q6_K", 4096, 12288, 8, 4],
                                        ["Q8_0", 1024, 1024, 2, 2], ["Q5_K", 5120, 10240, 8, 1]]},
    {"name": "collision_last_wins", "configs": [["Q4_K", 2048, 2048, 2, 2], ["Q4_K", 4096, 3000, 8, 4]]},
    {"name": "collision_priority", "configs": [["Q4_K", 2048, 2048, 2, 2], ["Q4_K", 4096, 3000, 8, 4]],
     "priorities": [["Q4_K", 2048, 2048, 1.5], ["Q4_K", 4096, 3000, 1.2]]},
    {"name": "priority_nan", "configs": [["Q4_K", 2048, 2048, 2, 2], ["Q4_K", 4096, 3000, 8, 4]],
     "priorities": [["Q4_K", 2048, 2048, 1.1], ["Q4_K", 4096, 3000, "nan"]]},
    {"name": "unknown_type", "configs": [["F16", 4096, 4096, 8, 2], ["Q4_K", 151936, 4096, 1, 4]]},
]

MERGE_CASES = [
    {"name": "disjoint", "payloads": [
        {"gpu": "b200", "model": "a", "configs": {"12": {"2,2": {"nwarps": 8, "rows_per_block": 2}}}},
        {"gpu": "x", "model": "b", "configs": {"8": {"1,1": {"nwarps": 2, "rows_per_block": 1}}}}]},
    {"name": "conflict_first_wins", "payloads": [
        {"gpu": "g", "model": "t", "configs": {"12": {"2,2": {"nwarps": 8, "rows_per_block": 2}}}},
        {"gpu": "g", "model": "d", "configs": {"12": {"2,2": {"nwarps": 1, "rows_per_block": 4},
                                                     "3,2": {"nwarps": 2, "rows_per_block": 2}}}}]},
    {"name": "malformed", "payloads": [
        "not a dict", {"gpu": 5, "model": None, "configs": "oops"},
        {"model": "ok", "configs": {"12": None, "13": "x", "14": {"1,1": 7, "2,2": {"nwarps": 4}}}}]},
    {"name": "empty", "payloads": []},
]

SMITHY_DOCS = {
    "basic": '{"gpu":"b200","model":"m","configs":{"12":{"2,2":{"nwarps":8,"rows_per_block":2},'
             '"3,2":{"nwarps":4,"rows_per_block":4}},"14":{"1,2":{"nwarps":2,"rows_per_block":1}}}}',
    "clamp": '{"configs":{"12":{"0,0":{"nwarps":33,"rows_per_block":2},"1,1":{"nwarps":0,"rows_per_block":1},'
             '"2,2":{"nwarps":32,"rows_per_block":32},"3,3":{"nwarps":-1,"rows_per_block":2}}}}',
    "brace_in_string": '{"configs":{"12":{"comment":"see } here","2,2":{"nwarps":8,"rows_per_block":2}},'
                       '"13":{"1,1":{"nwarps":2,"rows_per_block":2}}}}',
    "string_value_type": '{"configs":{"12":"oops","13":{"2,2":{"nwarps":8,"rows_per_block":2}}}}',
    "string_value_cell": '{"configs":{"12":{"2,2":"oops","3,3":{"nwarps":4,"rows_per_block":2}}}}',
    "sibling_top_level": '{"configs":{"12":{"2,2":{"nwarps":8,"rows_per_block":2}}},'
                         '"telemetry":{"5":{"2,2":{"nwarps":3,"rows_per_block":3}}}}',
    "out_of_range_type": '{"configs":{"99":{"2,2":{"nwarps":8,"rows_per_block":2}},'
                         '"12":{"1,1":{"nwarps":2,"rows_per_block":2}}}}',
    "nested_digit_in_oor": '{"configs":{"77":{"3":{"2,2":{"nwarps":6,"rows_per_block":3}}}}}',
    "bad_bucket": '{"configs":{"12":{"5,1":{"nwarps":8,"rows_per_block":2},"1,-1":{"nwarps":8,"rows_per_block":2},'
                  '"4,4":{"nwarps":7,"rows_per_block":3}}}}',
    "whitespace": '{\n  "configs" : {\n    "12" : {\n      "2, 3" : { "nwarps" : 8 , "rows_per_block" : 2 }\n    }\n  }\n}',
    "float_and_string_values": '{"configs":{"12":{"2,2":{"nwarps":8.9,"rows_per_block":"2"},'
                               '"1,1":{"nwarps":4.2,"rows_per_block":2.7}}}}',
    "missing_field": '{"configs":{"12":{"2,2":{"nwarps":8},"3,3":{"rows_per_block":2,"nwarps":5}}}}',
    "no_configs": '{"gpu":"b200","model":"m"}',
    "configs_not_object": '{"configs":[1,2,3]}',
    "duplicate_cells": '{"configs":{"12":{"2,2":{"nwarps":8,"rows_per_block":2},"2,2":{"nwarps":4,"rows_per_block":4}}}}',
    "nested_in_cell": '{"configs":{"12":{"2,2":{"inner":{"nwarps":6,"rows_per_block":2}}}}}',
    "unterminated": '{"configs":{"12":{"2,2":{"nwarps":8,"rows_per_block":2}',
    "escaped_quotes": '{"configs":{"12":{"note":"a \\"2,2\\": {x}","3,3":{"nwarps":2,"rows_per_block":4}}}}',
    "generated_by_codegen": None,  # filled from the reference's generate_runtime_config
}


def write_dequant(out: Path, types=None) -> None:
    import gguf

    for qt, (n, k) in DEQUANT_CASES.items():
        if types and qt not in types:
            continue
        W = make_weights(qt, n, k, seed=11)
        deq = gguf.quants.dequantize(W, getattr(gguf.GGMLQuantizationType, qt))
        np.savez_compressed(out / f"dequant_{qt}.npz", W=W, dequant=deq.astype(np.float32),
                            nrows=n, K=k)
    if types:
        return
    x = make_activation(1024, ncols=2, seed=5)
    x[1, :32] = 0.0  # an all-zero block
    q8 = gguf.quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    np.savez_compressed(out / "q8_0_gguf.npz", x=x, q8_0=q8)


_CODEGEN_DRIVER = r'''
import json, sys
from kernel_anvil import codegen
cases = json.load(sys.stdin)
res = {"bucket_index": {str(v): codegen.bucket_index(v) for v in
       [0, 1, 64, 128, 129, 500, 1024, 1025, 2048, 4096, 4097, 8192, 16384, 16385, 151936]},
       "runtime": {}, "header": {}, "merge": {}}
for c in cases["codegen"]:
    cfgs = {(q, n, k): {"nwarps": nw, "rows_per_block": r} for q, n, k, nw, r in c["configs"]}
    pri = None
    if "priorities" in c:
        pri = {(q, n, k): float(p) for q, n, k, p in c["priorities"]}
    res["runtime"][c["name"]] = codegen.generate_runtime_config(cfgs, gpu_name="b200", model_name=c["name"], priorities=pri)
    res["header"][c["name"]] = codegen.generate_config_header(cfgs, gpu_name="b200", model_name=c["name"])
for m in cases["merge"]:
    res["merge"][m["name"]] = codegen.merge_runtime_configs(m["payloads"])
json.dump(res, sys.stdout)
'''


def write_codegen(out: Path, reference: Path) -> dict:
    env = dict(os.environ, PYTHONPATH=str(reference))
    payload = json.dumps({"codegen": CODEGEN_CASES, "merge": MERGE_CASES})
    r = subprocess.run([sys.executable, "-c", _CODEGEN_DRIVER], input=payload, capture_output=True,
                       text=True, env=env, cwd=tempfile.gettempdir(), check=True)
    res = json.loads(r.stdout)
    # The header carries a generation timestamp; tests compare everything else.
    for name, text in res["header"].items():
        res["header"][name] = "\n".join(
            "// Generated: <timestamp>" if ln.startswith("// Generated: ") else ln for ln in text.split("\n"))
    (out / "codegen.json").write_text(json.dumps({"cases": CODEGEN_CASES, "merge_cases": MERGE_CASES,
                                                  "results": res}, indent=1, sort_keys=True))
    return res


def write_smithy(out: Path, codegen_res: dict) -> None:
    sys.path.insert(0, str(REPO))
    from oracle import oracle

    ref = oracle.ref_smithy()
    if ref is None:
        raise SystemExit("oracle/_ref/libsmithy_ref.so is missing (make -C oracle with the reference tree)")
    docs = dict(SMITHY_DOCS)
    docs["generated_by_codegen"] = codegen_res["runtime"]["multi_type"]
    results = {}
    with tempfile.TemporaryDirectory() as td:
        for name, text in docs.items():
            p = Path(td) / f"{name}.json"
            p.write_text(text)
            ref.ref_smithy_clear()
            ok = ref.ref_smithy_load(str(p).encode())
            cells = []
            nw, rpb = ctypes.c_int(), ctypes.c_int()
            for t in range(41):
                for nb in range(5):
                    for kb in range(5):
                        ref.ref_smithy_cell(t, nb, kb, ctypes.byref(nw), ctypes.byref(rpb))
                        if nw.value or rpb.value:
                            cells.append([t, nb, kb, nw.value, rpb.value])
            results[name] = {"doc": text, "ok": bool(ok), "loaded": bool(ref.ref_smithy_loaded()),
                             "cells": cells}
    (out / "smithy_loader.json").write_text(json.dumps(results, indent=1, sort_keys=True))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--types", nargs="*", default=None,
                    help="only the dequant fixtures of these types (nothing else is rewritten)")
    args = ap.parse_args()
    write_dequant(HERE, args.types)
    if args.types:
        print(f"dequant fixtures of {' '.join(args.types)} written to {HERE}")
        return
    res = write_codegen(HERE, Path(args.reference))
    write_smithy(HERE, res)
    print(f"fixtures written to {HERE}")


if __name__ == "__main__":
    main()
