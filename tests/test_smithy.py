"""libanvil's smithy loader (anvil_smithy_*) against the reference's own loader.

The reference loader is patches/smithy-config.h.  Its tables on a battery of documents,
malformed ones included, are frozen in tests/golden/smithy_loader.json (make_golden.py).
When oracle/_ref/libsmithy_ref.so exists (the header compiled in place by oracle/Makefile),
random documents are also compared live.  Lookup precedence follows
patches/smithy-config.h:268-317 and is exercised with HOME and env vars sandboxed.
"""
import ctypes
import json
from pathlib import Path
import random
import threading

import pytest

from kernel_anvil import _native
from kernel_anvil.codegen import bucket_index, generate_runtime_config
from oracle import oracle

lib = _native.lib()


def table_cells(loader_lookup) -> list[list[int]]:
    cells = []
    nw, rpb = ctypes.c_int(), ctypes.c_int()
    reps = [64, 512, 2048, 8192, 100000]  # one representative dimension per bucket
    for t in range(41):
        for nb in range(5):
            for kb in range(5):
                loader_lookup(t, reps[nb], reps[kb], ctypes.byref(nw), ctypes.byref(rpb))
                if nw.value or rpb.value:
                    cells.append([t, nb, kb, nw.value, rpb.value])
    return cells


def anvil_load_doc(tmp_path, text: str, name="doc.json"):
    p = tmp_path / name
    p.write_text(text)
    lib.anvil_smithy_reset()
    n = lib.anvil_smithy_load(str(p).encode())
    return n, table_cells(lib.anvil_smithy_lookup)


@pytest.fixture(autouse=True)
def clean_table(sandbox_home):
    lib.anvil_smithy_reset()
    yield
    lib.anvil_smithy_reset()


def test_bucket_boundaries_match_codegen():
    for v in [0, 1, 128, 129, 1024, 1025, 4096, 4097, 16384, 16385, 151936, -5]:
        assert lib.anvil_smithy_bucket(v) == bucket_index(v)


def test_golden_documents_match_reference(golden_dir, tmp_path):
    gold = json.loads((golden_dir / "smithy_loader.json").read_text())
    for name, case in gold.items():
        n, cells = anvil_load_doc(tmp_path, case["doc"], f"{name}.json")
        # lookups only see the table while it is marked loaded (>= 1 cell accepted)
        want = case["cells"] if case["loaded"] else []
        assert cells == want, name
        assert (n > 0) == case["loaded"] == case["ok"], name


def _random_doc(rng: random.Random) -> str:
    def cell():
        r = rng.random()
        if r < 0.1:
            return '"x"'
        nw = rng.choice([0, 1, 2, 4, 8, 16, 32, 33, -1, 7])
        rpb = rng.choice([0, 1, 2, 4, 32, 40])
        extra = ', "note": "}{"' if rng.random() < 0.2 else ""
        return f'{{"nwarps": {nw}, "rows_per_block": {rpb}{extra}}}'

    types = []
    for _ in range(rng.randint(0, 5)):
        t = rng.choice(["12", "13", "14", "8", "2", "40", "41", "99", "meta", "7x"])
        cells = []
        for _ in range(rng.randint(0, 6)):
            key = rng.choice([f"{rng.randint(-1, 5)},{rng.randint(-1, 5)}", "note", "2, 2", "3,1,9"])
            cells.append(f'"{key}": {cell()}')
        body = "{" + ", ".join(cells) + "}" if rng.random() > 0.1 else '"oops"'
        types.append(f'"{t}": {body}')
    doc = '{"gpu": "b200", "configs": {' + ", ".join(types) + '}, "model": "m"}'
    if rng.random() < 0.1:
        doc = doc[: rng.randint(1, len(doc))]
    return doc


def test_random_documents_match_live_reference(tmp_path):
    ref = oracle.ref_smithy()
    if ref is None:
        pytest.skip("oracle/_ref/libsmithy_ref.so not built (reference tree absent)")
    rng = random.Random(1234)
    for i in range(300):
        doc = _random_doc(rng)
        p = tmp_path / f"r{i}.json"
        p.write_text(doc)
        ref.ref_smithy_clear()
        ok = ref.ref_smithy_load(str(p).encode())
        ref_cells = table_cells(lambda t, n, k, a, b: ref.ref_smithy_cell(
            t, bucket_index(n), bucket_index(k), a, b)) if ok else []
        n, cells = anvil_load_doc(tmp_path, doc, f"a{i}.json")
        assert cells == ref_cells, doc
        assert (n > 0) == bool(ok), doc


def test_codegen_output_loads(tmp_path):
    cfgs = {("Q4_K", 4096, 4096): {"nwarps": 8, "rows_per_block": 2},
            ("Q6_K", 4096, 12288): {"nwarps": 2, "rows_per_block": 4}}
    n, cells = anvil_load_doc(tmp_path, generate_runtime_config(cfgs))
    assert n == 2
    assert [12, 2, 2, 8, 2] in cells and [14, 2, 3, 2, 4] in cells


def test_size_cap_and_missing_file(tmp_path):
    big = tmp_path / "big.json"
    big.write_text('{"configs": {"12": {"2,2": {"nwarps": 8, "rows_per_block": 2}}}}' + " " * (1 << 20))
    assert lib.anvil_smithy_load(str(big).encode()) < 0
    assert lib.anvil_smithy_load(str(tmp_path / "absent.json").encode()) < 0
    empty = tmp_path / "empty.json"
    empty.write_text("")
    assert lib.anvil_smithy_load(str(empty).encode()) < 0


def _write(path, cells):
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"configs": {"12": cells}}))


def lookup(n=4096, k=4096, t=12):
    nw, rpb = ctypes.c_int(), ctypes.c_int()
    found = lib.anvil_smithy_lookup(t, n, k, ctypes.byref(nw), ctypes.byref(rpb))
    return found, (nw.value, rpb.value)


def test_precedence_env_config_first(sandbox_home, monkeypatch, tmp_path):
    cache = sandbox_home / ".cache" / "smithy"
    _write(cache / "default.json", {"2,2": {"nwarps": 1, "rows_per_block": 1}})
    _write(cache / "Qwen3-8B-Q4_K_M.json", {"2,2": {"nwarps": 2, "rows_per_block": 2}})
    _write(tmp_path / "explicit.json", {"2,2": {"nwarps": 8, "rows_per_block": 4}})
    monkeypatch.setenv("SMITHY_CONFIG", str(tmp_path / "explicit.json"))
    lib.anvil_smithy_set_model(b"/models/Qwen3-8B-Q4_K_M.gguf")
    assert lookup() == (1, (8, 4))


def test_precedence_model_stem_then_default(sandbox_home, monkeypatch):
    cache = sandbox_home / ".cache" / "smithy"
    _write(cache / "default.json", {"2,2": {"nwarps": 1, "rows_per_block": 1}})
    _write(cache / "Qwen3-8B-Q4_K_M.json", {"2,2": {"nwarps": 2, "rows_per_block": 2}})
    monkeypatch.setenv("SMITHY_CONFIG", str(sandbox_home / "nope.json"))  # unreadable: skipped
    lib.anvil_smithy_set_model(b"/models/Qwen3-8B-Q4_K_M.gguf")
    assert lookup() == (1, (2, 2))
    lib.anvil_smithy_set_model(b"C:\\models\\other.gguf")  # unknown stem -> default.json
    assert lookup() == (1, (1, 1))


def test_precedence_smithy_model_env(sandbox_home, monkeypatch):
    cache = sandbox_home / ".cache" / "smithy"
    _write(cache / "tiny.json", {"1,1": {"nwarps": 4, "rows_per_block": 8}})
    monkeypatch.setenv("SMITHY_MODEL", "/x/y/tiny.q4.gguf".replace(".q4", ""))
    lib.anvil_smithy_reset()
    assert lookup(512, 512) == (1, (4, 8))
    assert lookup(4096, 4096) == (0, (0, 0))  # cell absent: no override


def test_no_config_anywhere_means_no_override(sandbox_home):
    assert lookup() == (0, (0, 0))
    assert lib.anvil_smithy_try_load() == 0


def test_concurrent_lookups_and_resets(sandbox_home, tmp_path, monkeypatch):
    _write(tmp_path / "c.json", {"2,2": {"nwarps": 8, "rows_per_block": 2}})
    monkeypatch.setenv("SMITHY_CONFIG", str(tmp_path / "c.json"))
    lib.anvil_smithy_reset()
    bad = []

    def reader():
        for _ in range(3000):
            found, v = lookup()
            if v not in ((8, 2), (0, 0)):
                bad.append(v)

    def writer():
        for _ in range(200):
            lib.anvil_smithy_set_model(b"/m/c.gguf")

    ts = [threading.Thread(target=reader) for _ in range(4)] + [threading.Thread(target=writer)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not bad


TUNED = Path(__file__).resolve().parent.parent / "kernel-anvil_b200" / "kernel_anvil" / "tuned"


@pytest.mark.parametrize("name,types", [("smithy_qwen3_8b_plus_draft.json", {8, 12, 14}),
                                        ("smithy_qwen35_27b.json", {12, 13}),
                                        ("tuned:llama3_70b_b200.json", {12})])
def test_recorded_tuner_outputs_load_like_the_reference(golden_dir, tmp_path, name, types):
    """Configs the tuner wrote on a B200 (gguf-optimize with a draft model; autoforge on the
    Qwen3.5-27B and Llama-3-70B shapes, the latter shipped for the bench) load with the same
    cells in this loader and in the reference's."""
    if name.startswith("tuned:"):
        name = name[len("tuned:"):]
        doc = (TUNED / name).read_text()
    else:
        doc = (golden_dir / name).read_text()
    n, cells = anvil_load_doc(tmp_path, doc, name)
    assert n > 0 and {c[0] for c in cells} == types
    ref = oracle.ref_smithy()
    if ref is None:
        pytest.skip("oracle/_ref/libsmithy_ref.so not built (reference tree absent)")
    p = tmp_path / f"ref_{name}"
    p.write_text(doc)
    ref.ref_smithy_clear()
    assert ref.ref_smithy_load(str(p).encode())
    ref_cells = table_cells(lambda t, n_, k, a, b: ref.ref_smithy_cell(
        t, bucket_index(n_), bucket_index(k), a, b))
    assert cells == ref_cells
