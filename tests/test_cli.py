"""The kernel-anvil CLI on CPU: argument handling, merge-configs, gguf-optimize on synthetic
GGUF files (--no-bench, --draft merging, --legacy-keys, failed shapes, header output), and
the ncu CSV parser.  Mirrors the reference's tests/test_cli*.py and test_gguf_optimize*.py
expectations; GPU tuning itself is covered by tests/test_gpu_cli.py."""
import json
from pathlib import Path
from types import SimpleNamespace

import pytest

from kernel_anvil import cli
from kernel_anvil.codegen import GGML_TYPE_MAP, bucket_index, generate_runtime_config
from kernel_anvil.gguf import parse_gguf, write_gguf


def _run(argv):
    with pytest.raises(SystemExit) as e:
        cli.main(argv)
    return e.value.code


def _model(tmp_path, name, tensors, seed=0):
    return write_gguf(tmp_path / f"{name}.gguf", tensors, name=name, seed=seed)


TARGET = [("blk.0.attn_q.weight", "Q4_K", 256, 512),
          ("blk.0.ffn_down.weight", "Q6_K", 512, 1024),
          ("blk.1.attn_q.weight", "Q4_K", 256, 512),
          ("blk.0.attn_norm.weight", "F32", 1, 512),
          ("output.weight", "Q8_0", 320, 256)]


def test_no_command_prints_help_and_exits_1(capsys):
    assert _run([]) == 1
    assert "gguf-optimize" in capsys.readouterr().out


@pytest.mark.parametrize("sub", ["sweep", "profile", "gguf-optimize", "merge-configs", "autoforge",
                                 "chain-sweep", "bench-gemv"])
def test_subcommand_help(sub, capsys):
    assert _run([sub, "--help"]) == 0
    assert "usage" in capsys.readouterr().out


def test_reference_defaults():
    p = cli.build_parser()
    a = p.parse_args(["gguf-optimize", "m.gguf"])
    assert (a.output, a.max_configs, a.warmup, a.runs, a.no_bench, a.draft, a.legacy_keys) == \
        ("smithy-config.h", 15, 3, 5, False, None, False)
    a = p.parse_args(["sweep", "r.py"])
    assert (a.max_configs, a.warmup, a.runs, a.atol, a.rtol) == (20, 5, 10, 1e-2, 1e-2)
    a = p.parse_args(["profile", "r.py"])
    assert (a.warmup, a.runs) == (5, 20)
    a = p.parse_args(["autoforge", "m.gguf"])
    assert (a.nwarps, a.rpb) == ("1,2,4,8", "1,2,4")
    a = p.parse_args(["gguf-optimize", "t.gguf", "--draft", "a.gguf", "--draft", "b.gguf"])
    assert a.draft == ["a.gguf", "b.gguf"]


# ---------------------------------------------------------------------------------------
# merge-configs
# ---------------------------------------------------------------------------------------

def _write(p: Path, obj) -> Path:
    p.write_text(json.dumps(obj))
    return p


def test_merge_configs_first_wins(tmp_path):
    a = _write(tmp_path / "a.json", {"gpu": "sm_100a", "model": "A",
                                     "configs": {"12": {"0,0": {"nwarps": 2, "rows_per_block": 1}}}})
    b = _write(tmp_path / "b.json", {"gpu": "x", "model": "B",
                                     "configs": {"12": {"0,0": {"nwarps": 8, "rows_per_block": 4},
                                                        "1,1": {"nwarps": 1, "rows_per_block": 2}},
                                                 "14": {"2,2": {"nwarps": 4, "rows_per_block": 2}}}})
    out = tmp_path / "sub" / "m.json"
    cli.main(["merge-configs", str(a), str(b), "-o", str(out)])
    m = json.loads(out.read_text())
    assert m == {"gpu": "sm_100a", "model": "A+B",
                 "configs": {"12": {"0,0": {"nwarps": 2, "rows_per_block": 1},
                                    "1,1": {"nwarps": 1, "rows_per_block": 2}},
                             "14": {"2,2": {"nwarps": 4, "rows_per_block": 2}}}}
    assert [p.name for p in out.parent.iterdir()] == ["m.json"]  # no temp file left behind


def test_merge_configs_overrides(tmp_path):
    a = _write(tmp_path / "a.json", {"gpu": "g", "model": "A", "configs": {}})
    out = tmp_path / "m.json"
    cli.main(["merge-configs", str(a), "-o", str(out), "--gpu", "sm_100a", "--model", "both"])
    assert json.loads(out.read_text())[("gpu")] == "sm_100a"
    assert json.loads(out.read_text())["model"] == "both"


def test_merge_configs_missing_input(tmp_path):
    out = tmp_path / "m.json"
    assert _run(["merge-configs", str(tmp_path / "nope.json"), "-o", str(out)]) == 1
    assert not out.exists()


def test_merge_configs_invalid_json(tmp_path):
    bad = tmp_path / "bad.json"
    bad.write_text("{not json")
    out = tmp_path / "m.json"
    out.write_text("previous")
    assert _run(["merge-configs", str(bad), "-o", str(out)]) == 1
    assert out.read_text() == "previous"


# ---------------------------------------------------------------------------------------
# gguf-optimize
# ---------------------------------------------------------------------------------------

def _cache(home: Path, stem: str) -> dict:
    return json.loads((home / ".cache" / "smithy" / f"{stem}.json").read_text())


def test_gguf_optimize_no_bench(tmp_path, sandbox_home):
    m = _model(tmp_path, "tiny", TARGET)
    cli.main(["gguf-optimize", str(m), "--no-bench"])
    got = _cache(sandbox_home, "tiny")
    # every shape gets the built-in launch; 2-D F32 would be skipped, the 1-D norm is no GEMV
    want = {("Q4_K", 256, 512): cli.heuristic_config("Q4_K", 256, 512),
            ("Q6_K", 512, 1024): cli.heuristic_config("Q6_K", 512, 1024),
            ("Q8_0", 320, 256): cli.heuristic_config("Q8_0", 320, 256)}
    assert got == json.loads(generate_runtime_config(want, gpu_name="sm_100a", model_name="tiny"))
    assert got["configs"][str(GGML_TYPE_MAP["Q6_K"])] == {
        f"{bucket_index(512)},{bucket_index(1024)}": {"nwarps": 8, "rows_per_block": 1}}


def test_gguf_optimize_falls_back_without_gpu(tmp_path, sandbox_home, monkeypatch):
    monkeypatch.setattr(cli, "_gpu_available", lambda: False)
    m = _model(tmp_path, "fb", TARGET[:1])
    cli.main(["gguf-optimize", str(m)])
    assert _cache(sandbox_home, "fb")["configs"]


def test_gguf_optimize_missing_files(tmp_path, sandbox_home):
    assert _run(["gguf-optimize", str(tmp_path / "no.gguf"), "--no-bench"]) == 1
    m = _model(tmp_path, "t", TARGET[:1])
    assert _run(["gguf-optimize", str(m), "--draft", str(tmp_path / "no.gguf"), "--no-bench"]) == 1
    assert not (sandbox_home / ".cache" / "smithy" / "t.json").exists()


def test_gguf_optimize_no_weights(tmp_path, sandbox_home):
    m = _model(tmp_path, "empty", [("norm.weight", "F32", 1, 64)])
    assert _run(["gguf-optimize", str(m), "--no-bench"]) == 0
    assert not (sandbox_home / ".cache" / "smithy" / "empty.json").exists()


def test_gguf_optimize_header_and_legacy_keys(tmp_path, sandbox_home):
    m = _model(tmp_path, "hdr", [("a.weight", "Q4_K", 4096, 256)])
    hdr = tmp_path / "out.h"
    cli.main(["gguf-optimize", str(m), "--no-bench", "--legacy-keys", "--output", str(hdr)])
    text = hdr.read_text()
    assert "smithy" in text.lower() and "hdr" in text
    cells = _cache(sandbox_home, "hdr")["configs"][str(GGML_TYPE_MAP["Q4_K"])]
    # legacy key: (ne0, ne1) = (K cols, N rows) -> buckets of (256, 4096)
    assert list(cells) == [f"{bucket_index(256)},{bucket_index(4096)}"]
    # the heuristic still sees the true shape (N=4096 rows, K=256)
    assert cells[list(cells)[0]] == cli.heuristic_config("Q4_K", 4096, 256)


def _args(**kw):
    base = dict(max_configs=15, warmup=3, runs=5, no_bench=False, draft=None, legacy_keys=False,
                output="smithy-config.h")
    base.update(kw)
    return SimpleNamespace(**base)


def test_gguf_optimize_draft_priorities_and_failed_shapes(tmp_path, sandbox_home):
    """Target and draft share a bucket cell: the shape with the higher speedup owns it.  A
    target shape whose tuning failed is absent from the table, so the draft's run of the same
    shape fills it (cli.py:338-409 of the reference)."""
    target = _model(tmp_path, "big", [("a.weight", "Q4_K", 4096, 4096),
                                      ("b.weight", "Q6_K", 1024, 1024)])
    draft = _model(tmp_path, "small", [("c.weight", "Q4_K", 3840, 3840),
                                       ("d.weight", "Q6_K", 1024, 1024)], seed=5)
    calls = []

    def fake_tune(quant, n, k, max_configs, warmup, runs):
        calls.append((quant, n, k))
        if (quant, n, k) == ("Q6_K", 1024, 1024) and calls.count((quant, n, k)) == 1:
            raise RuntimeError("launch failed")
        table = {("Q4_K", 4096, 4096): ({"nwarps": 2, "rows_per_block": 2}, 10.0, 1.1),
                 ("Q4_K", 3840, 3840): ({"nwarps": 8, "rows_per_block": 4}, 10.0, 1.6),
                 ("Q6_K", 1024, 1024): ({"nwarps": 1, "rows_per_block": 2}, 5.0, 1.3)}
        return table[(quant, n, k)]

    cli.cmd_gguf_optimize(_args(gguf=str(target), draft=[str(draft)]), tune=fake_tune)
    assert calls == [("Q4_K", 4096, 4096), ("Q6_K", 1024, 1024), ("Q4_K", 3840, 3840),
                     ("Q6_K", 1024, 1024)]
    got = _cache(sandbox_home, "big")
    assert got["model"] == "big+small"
    q4 = got["configs"][str(GGML_TYPE_MAP["Q4_K"])]
    assert q4 == {f"{bucket_index(4096)},{bucket_index(4096)}": {"nwarps": 8, "rows_per_block": 4}}
    q6 = got["configs"][str(GGML_TYPE_MAP["Q6_K"])]
    assert q6 == {f"{bucket_index(1024)},{bucket_index(1024)}": {"nwarps": 1, "rows_per_block": 2}}
    assert not (sandbox_home / ".cache" / "smithy" / "small.json").exists()


def test_gguf_optimize_shared_shape_reused(tmp_path, sandbox_home):
    target = _model(tmp_path, "t2", [("a.weight", "Q4_K", 512, 512)])
    draft = _model(tmp_path, "d2", [("b.weight", "Q4_K", 512, 512)], seed=3)
    calls = []

    def fake_tune(quant, n, k, *rest):
        calls.append((quant, n, k))
        return {"nwarps": 2, "rows_per_block": 1}, 3.0, 1.2

    cli.cmd_gguf_optimize(_args(gguf=str(target), draft=[str(draft)]), tune=fake_tune)
    assert calls == [("Q4_K", 512, 512)]


def test_parse_gguf_roundtrip_shapes(tmp_path):
    m = _model(tmp_path, "shapes", TARGET)
    prof = parse_gguf(m)
    assert prof.unique_shapes[("Q4_K", 512, 256)] == 2          # (ne0, ne1) = (K, N)
    assert prof.gemv_shapes()[("Q4_K", 256, 512)] == 2           # (N, K)


# ---------------------------------------------------------------------------------------
# runner / autoforge argument errors, ncu CSV parsing
# ---------------------------------------------------------------------------------------

def test_sweep_missing_runner(tmp_path):
    assert _run(["sweep", str(tmp_path / "none.py")]) == 1
    assert _run(["profile", str(tmp_path / "none.py")]) == 1


def test_runner_without_reference(tmp_path):
    r = tmp_path / "r.py"
    r.write_text("def setup():\n    return None\n\ndef run(inputs, **cfg):\n    return None\n")
    assert _run(["sweep", str(r)]) == 1


def test_autoforge_bad_values(tmp_path):
    assert _run(["autoforge", "--chain", "qwen3_8b", "--nwarps", "0,4"]) == 1
    assert _run(["autoforge"]) == 1
    assert _run(["autoforge", str(tmp_path / "none.gguf")]) == 1


def test_parse_ncu_csv():
    from kernel_anvil.profile import parse_ncu_csv

    text = "\n".join([
        "==PROF== Connected to process 1",
        '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
        '"Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit",'
        '"Metric Value"',
        '"0","1","python","h","void mmvq_kernel<12, 1, 4, 0, 16>(MmvqArgs)","1","7","(128, 1, 1)",'
        '"(296, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","Mbyte",'
        '"17.10"',
        '"0","1","python","h","void mmvq_kernel<12, 1, 4, 0, 16>(MmvqArgs)","1","7","(128, 1, 1)",'
        '"(296, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum",'
        '"usecond","7,25"'.replace("7,25", "7.25"),
        '"1","1","python","h","void quantize_q8_1_kernel(const float*)","1","7","(256, 1, 1)",'
        '"(4, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum",'
        '"nsecond","1500"',
    ])
    rows = parse_ncu_csv(text)
    assert rows[0]["kernel"] == "mmvq_kernel<12, 1, 4, 0, 16>"
    assert rows[0]["dram__bytes_read.sum"] == pytest.approx(17.10e6)
    assert rows[0]["gpu__time_duration.sum"] == pytest.approx(7.25)
    assert rows[1]["gpu__time_duration.sum"] == pytest.approx(1.5)
    assert parse_ncu_csv("no csv here") == []


GOLDEN = Path(__file__).parent / "golden"


def test_recorded_ncu_capture_parses_to_per_launch_metrics():
    """tests/golden/ncu_mmvq_q4k_12288x4096.csv: three launches of the Q4_K 12288 x 4096 MMVQ
    kernel under ncu (one pass of gpu__time_duration and DRAM bytes, clocks left alone)."""
    from kernel_anvil.analyze import ProfileMetrics
    from kernel_anvil.profile import apply_ncu, parse_ncu_csv
    from kernel_anvil.quants import gemv_bytes

    rows = parse_ncu_csv((GOLDEN / "ncu_mmvq_q4k_12288x4096.csv").read_text())
    assert len(rows) == 3 and all(r["kernel"].startswith("mmvq_kernel<12, 1") for r in rows)
    m = apply_ncu(ProfileMetrics(duration_ns=0.0), rows)
    # DRAM reads are the weight bytes (plus the small activation): no re-reads
    assert m.dram_bytes == pytest.approx(gemv_bytes("Q4_K", 12288, 4096), rel=0.01)
    assert 9_000 < m.duration_ns < 12_000


def test_profile_cli_classifies_recorded_capture_as_bandwidth_bound(capsys, monkeypatch):
    """`kernel-anvil profile RUNNER --ncu-csv CSV` on a host without a GPU: the recorded capture
    of the Q4_K 28672 x 8192 GEMV (132 MB read in about 27 us per cold launch) goes through
    parse -> apply_ncu -> classify and comes out bandwidth_bound."""
    import torch

    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    cli.main(["profile", str(GOLDEN / "runner_mmvq_q4k_28672x8192.py"),
              "--ncu-csv", str(GOLDEN / "ncu_mmvq_q4k_28672x8192.csv")])
    out = capsys.readouterr().out
    assert "Classification: bandwidth_bound" in out


def test_write_gguf_chain_layers(tmp_path):
    """write-gguf: one decoder layer of a chain holds every unique GEMV shape of the chain."""
    from kernel_anvil.chains import get_chain

    out = tmp_path / "draft.gguf"
    cli.main(["write-gguf", "qwen3_0_6b", str(out), "--layers", "1"])
    prof = parse_gguf(out)
    assert set(prof.gemv_shapes()) == set(get_chain("qwen3_0_6b").unique_shapes())
    assert {t.name for t in prof.tensors} == {f"blk.0.{n}.weight" for n in (
        "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")}
    assert _run(["write-gguf", "no_such_chain", str(tmp_path / "x.gguf")]) == 1
    assert _run(["write-gguf", "qwen3_0_6b", str(tmp_path / "y.gguf"), "--layers", "0"]) == 1


def test_chain_tensors_keeps_tail_once():
    from kernel_anvil.chains import get_chain

    t = cli.chain_tensors(get_chain("qwen3_8b"), 2)
    assert sum(1 for n, *_ in t if n.startswith("blk.")) == 14
    assert [n for n, *_ in t if not n.startswith("blk.")] == ["output.weight"]
