"""bench.py's host-side helpers (no GPU): the roofline traffic it reads from the committed ncu
summaries, and the launch-shape table it loads through the smithy loader."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_traffic_lines_of_the_committed_summaries(bench):
    v, src = bench.traffic_per_launch("mmvq_kernel llama3_70b")
    assert v == pytest.approx(120498606) and "ncu" in src
    v, src = bench.traffic_per_launch("pchain_kernel llama3_70b x1")
    assert v == pytest.approx(39554796371) and "times the full token" in src
    assert bench.traffic_per_launch("no_such_kernel") == (None, None)


def test_launch_table_choices(bench, tmp_path):
    from kernel_anvil import _native

    lib = _native.lib()
    name = bench.load_launch_table("auto", "llama3_70b")
    assert name.startswith("llama3_70b_b200.json")
    nw, rpb = _native.ctypes.c_int(), _native.ctypes.c_int()
    # 28672 x 8192 Q4_K: the tuned cell (8 warps, 2-row tiles)
    assert lib.anvil_smithy_lookup(12, 28672, 8192, _native.ctypes.byref(nw), _native.ctypes.byref(rpb)) == 1
    assert (nw.value, rpb.value) == (8, 2)
    assert bench.load_launch_table("auto", "qwen3_8b") is None  # no tuned table shipped
    assert bench.load_launch_table("none", "llama3_70b") is None
    with pytest.raises(SystemExit):
        bench.load_launch_table(str(tmp_path / "missing.json"), "llama3_70b")
    lib.anvil_smithy_reset()
