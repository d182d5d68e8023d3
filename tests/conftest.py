"""Shared pytest setup: import paths, the `gpu` marker, and seeded fixtures.

Tests marked ``gpu`` need a CUDA device and the built libanvil.so; everything else runs
on CPU (the oracle, host logic, config I/O, the C ABI's CPU-only entry points).
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO / "kernel-anvil_b200", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libanvil.so")


def pytest_collection_modifyitems(config, items):
    # A gpu-marked test on a machine without CUDA is a hard failure, not a skip, when the
    # run asked for gpu tests explicitly (-m gpu); otherwise gpu tests are skipped.
    try:
        import torch
        have_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_cuda = False
    markexpr = config.getoption("-m") or ""
    if have_cuda or markexpr.strip() == "gpu":
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


@pytest.fixture
def sandbox_home(tmp_path, monkeypatch):
    """HOME redirected to a temp dir (the smithy cache lives under $HOME/.cache/smithy)."""
    monkeypatch.setenv("HOME", str(tmp_path))
    monkeypatch.delenv("SMITHY_CONFIG", raising=False)
    monkeypatch.delenv("SMITHY_MODEL", raising=False)
    return tmp_path


os.environ.setdefault("PYTHONHASHSEED", "0")
