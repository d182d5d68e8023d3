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
