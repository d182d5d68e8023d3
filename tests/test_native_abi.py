"""libanvil.so loads and exports every entry point include/anvil.h declares (CPU only:
no compute call is made without a GPU)."""
import ctypes
import re

import pytest

from kernel_anvil import _native

HEADER = _native.INCLUDE / "anvil.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"\b(anvil_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_core_entry_points():
    names = declared_functions()
    for must in ("anvil_quantize_q8_1", "anvil_mmvq", "anvil_mmvq_block_sums", "anvil_smithy_lookup",
                 "anvil_smithy_set_model", "anvil_chain_instantiate", "anvil_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"libanvil.so lacks {missing}"


def test_python_signatures_cover_header():
    # every declared function has a ctypes signature in kernel_anvil._native
    assert set(declared_functions()) <= set(_native.SIGNATURES)


def test_cpu_safe_entry_points():
    lib = _native.lib()
    assert lib.anvil_abi_version() == 2
    qk, nb = ctypes.c_int(), ctypes.c_int()
    expect = {2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
              10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210),
              20: (32, 18), 23: (256, 136), 16: (256, 66), 17: (256, 74), 22: (256, 82),
              18: (256, 98), 21: (256, 110), 19: (256, 50), 29: (256, 56)}
    for t, (q, b) in expect.items():
        assert lib.anvil_type_geometry(t, ctypes.byref(qk), ctypes.byref(nb)) == 0
        assert (qk.value, nb.value) == (q, b)
    # Q8_K (15) and I8 (24) have no MMVQ block geometry here
    for t in (15, 24):
        assert lib.anvil_type_geometry(t, ctypes.byref(qk), ctypes.byref(nb)) == _native.ANVIL_ERR_UNSUPPORTED
    assert "no block geometry" in _native.last_error()
    assert lib.anvil_row_bytes(12, 4096) == 16 * 144
    assert lib.anvil_row_bytes(14, 12288) == 48 * 210
    assert lib.anvil_row_bytes(12, 4000) == _native.ANVIL_ERR_INVALID
    # the device wait bound: host state only, no launch
    assert lib.anvil_get_wait_limit_ns() == 2_000_000_000
    assert lib.anvil_set_wait_limit_ns(10_000_000) == 0
    assert lib.anvil_get_wait_limit_ns() == 10_000_000
    assert lib.anvil_set_wait_limit_ns(61_000_000_000) == _native.ANVIL_ERR_INVALID
    assert lib.anvil_set_wait_limit_ns(0) == 0
    assert lib.anvil_get_wait_limit_ns() == 2_000_000_000


def test_check_raises_with_message():
    lib = _native.lib()
    with pytest.raises(_native.AnvilError, match="multiple of 256"):
        _native.check(lib.anvil_row_bytes(12, 100))


def test_built_for_sm100a():
    # the build flags request sm_100a code only (no PTX JIT, no other arch)
    assert _native.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
