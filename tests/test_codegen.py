"""kernel_anvil.codegen: byte-identical to the reference's codegen on the golden cases,
plus the reference's own unit-test expectations (tests/test_codegen.py there)."""
import json
import math

import pytest

from kernel_anvil.codegen import (BUCKET_BOUNDARIES, DEFAULT_CONFIG, GGML_TYPE_COUNT, GGML_TYPE_MAP,
                                  NUM_BUCKETS, ShapeConfig, bucket_index, build_config_tables,
                                  generate_config_header, generate_runtime_config,
                                  merge_runtime_configs)


@pytest.fixture(scope="module")
def gold(golden_dir):
    return json.loads((golden_dir / "codegen.json").read_text())


def _cfgs(case):
    return {(q, n, k): {"nwarps": nw, "rows_per_block": r} for q, n, k, nw, r in case["configs"]}


def _pri(case):
    if "priorities" not in case:
        return None
    return {(q, n, k): float(p) for q, n, k, p in case["priorities"]}


def test_bucket_index_golden(gold):
    for v, b in gold["results"]["bucket_index"].items():
        assert bucket_index(int(v)) == b


def test_runtime_config_golden(gold):
    for case in gold["cases"]:
        got = generate_runtime_config(_cfgs(case), gpu_name="b200", model_name=case["name"],
                                      priorities=_pri(case))
        assert got == gold["results"]["runtime"][case["name"]], case["name"]


def test_header_golden(gold):
    for case in gold["cases"]:
        got = generate_config_header(_cfgs(case), gpu_name="b200", model_name=case["name"])
        lines = ["// Generated: <timestamp>" if ln.startswith("// Generated: ") else ln
                 for ln in got.split("\n")]
        assert "\n".join(lines) == gold["results"]["header"][case["name"]], case["name"]


def test_merge_golden(gold):
    for case in gold["merge_cases"]:
        assert merge_runtime_configs(case["payloads"]) == gold["results"]["merge"][case["name"]]


class TestBucketIndex:
    def test_boundaries(self):
        for i, b in enumerate(BUCKET_BOUNDARIES):
            assert bucket_index(b) == i
            assert bucket_index(b + 1) == i + 1

    def test_large(self):
        assert bucket_index(151936) == NUM_BUCKETS - 1


class TestTables:
    def test_empty(self):
        assert build_config_tables({}) == {}

    def test_defaults_fill(self):
        t = build_config_tables({("Q4_K", 4096, 4096): {"nwarps": 8, "rows_per_block": 2}})["Q4_K"]
        assert t[2][2] == ShapeConfig(8, 2)
        assert sum(c == DEFAULT_CONFIG for row in t for c in row) == NUM_BUCKETS ** 2 - 1

    def test_priority_nan_never_wins(self):
        cfgs = {("Q4_K", 2048, 2048): {"nwarps": 2, "rows_per_block": 2},
                ("Q4_K", 4096, 3000): {"nwarps": 8, "rows_per_block": 4}}
        t = build_config_tables(cfgs, priorities={("Q4_K", 2048, 2048): 1.1,
                                                  ("Q4_K", 4096, 3000): math.nan})["Q4_K"]
        assert t[2][2] == ShapeConfig(2, 2)

    def test_frozen(self):
        with pytest.raises(AttributeError):
            DEFAULT_CONFIG.nwarps = 2


class TestRuntimeJson:
    def test_default_cells_omitted(self):
        out = json.loads(generate_runtime_config({("Q4_K", 4096, 4096): {"nwarps": 4, "rows_per_block": 1}}))
        assert out["configs"] == {}

    def test_type_ids(self):
        out = json.loads(generate_runtime_config({("Q6_K", 4096, 12288): {"nwarps": 8, "rows_per_block": 2}}))
        assert out["configs"] == {"14": {"2,3": {"nwarps": 8, "rows_per_block": 2}}}
        assert GGML_TYPE_MAP["Q4_K"] == 12 and GGML_TYPE_COUNT == 41


class TestMerge:
    def test_first_seen_wins(self):
        a = {"gpu": "g", "model": "t", "configs": {"12": {"2,2": {"nwarps": 8, "rows_per_block": 2}}}}
        b = {"gpu": "g", "model": "d", "configs": {"12": {"2,2": {"nwarps": 1, "rows_per_block": 1}}}}
        m = merge_runtime_configs([a, b])
        assert m["configs"]["12"]["2,2"]["nwarps"] == 8
        assert m["model"] == "t+d"

    def test_does_not_mutate(self):
        a = {"gpu": "g", "model": "t", "configs": {"12": {"2,2": {"nwarps": 8, "rows_per_block": 2}}}}
        snap = json.dumps(a, sort_keys=True)
        merge_runtime_configs([a])["configs"]["12"]["2,2"]["nwarps"] = 1
        assert json.dumps(a, sort_keys=True) == snap

    def test_overrides(self):
        m = merge_runtime_configs([{"configs": {}}], gpu_name="b200", model_name="x")
        assert (m["gpu"], m["model"]) == ("b200", "x")
