"""The CLI's GPU paths: gguf-optimize tuning the real kernels on a synthetic GGUF, and the
--no-bench launch matching the library's own built-in choice."""
import json

import pytest

from kernel_anvil import cli
from kernel_anvil.codegen import GGML_TYPE_MAP
from kernel_anvil.gguf import write_gguf

pytestmark = pytest.mark.gpu


def test_heuristic_matches_native_default():
    """--no-bench writes the launch the library itself picks when no table matches."""
    from kernel_anvil import mmvq as ops

    for n, k in ((256, 512), (4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)):
        p = ops.plan("Q4_K", n, k)
        want = cli.heuristic_config("Q4_K", n, k)
        assert (p["nwarps"], p["rows_per_block"]) == (want["nwarps"], want["rows_per_block"])


def test_gguf_optimize_tunes_real_kernels(tmp_path, sandbox_home):
    m = write_gguf(tmp_path / "tune.gguf", [("a.weight", "Q4_K", 2048, 1024),
                                             ("b.weight", "Q6_K", 512, 2048),
                                             ("c.weight", "Q8_0", 1024, 512)], name="tune")
    cli.main(["gguf-optimize", str(m), "--runs", "20"])
    got = json.loads((sandbox_home / ".cache" / "smithy" / "tune.json").read_text())
    assert got["gpu"] == "sm_100a" and got["model"] == "tune"
    for cells in got["configs"].values():
        for cell in cells.values():
            assert cell["nwarps"] in (1, 2, 4, 8) and cell["rows_per_block"] in (1, 2, 4)
    assert set(got["configs"]) <= {str(GGML_TYPE_MAP[q]) for q in ("Q4_K", "Q6_K", "Q8_0")}


def test_kernel_attributes_are_real():
    """Registers and spills of the compiled MMVQ kernels (cudaFuncGetAttributes), the numbers
    the reference only estimated."""
    from kernel_anvil import mmvq as ops

    for qt, n, k, c in (("Q4_K", 4096, 4096, 1), ("Q6_K", 4096, 12288, 1), ("Q8_0", 1024, 1024, 8)):
        a = ops.kernel_attributes(qt, n, k, c)
        assert 16 <= a["regs_per_thread"] <= 255, a
        assert a["local_bytes"] >= 0 and a["max_threads_per_block"] >= 32


def test_profile_runner_reports_real_resources(capsys):
    from pathlib import Path

    from kernel_anvil.analyze import classify
    from kernel_anvil.profile import profile_kernel
    from kernel_anvil.specs import B200

    runner = Path(__file__).parent / "golden" / "runner_mmvq_q4k.py"
    spec = __import__("importlib.util").util.spec_from_file_location("runner_q4k", runner)
    mod = __import__("importlib.util").util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    inputs = mod.setup()
    m = profile_kernel(lambda c: mod.run(inputs, **c), mod.BASELINE_CONFIG, mod.DATA_BYTES, B200)
    assert m.regs_per_thread > 0 and m.smem_bytes > 0
    # the reference's decision order on the real numbers (the deep shared-memory rings keep
    # occupancy low by design, which the order reports before bandwidth)
    assert classify(m, B200).classification in ("occupancy_limited_smem", "occupancy_limited_regs",
                                                "bandwidth_bound", "launch_overhead", "compute_bound")
    cli.main(["profile", str(runner), "--runs", "5"])
    assert "Registers/thread" in capsys.readouterr().out
