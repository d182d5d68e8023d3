"""Build and load libanvil.so, the sm_100a CUDA library behind every GPU op here.

The library is compiled in-tree (``kernel_anvil/_lib/libanvil.so``) from ``csrc/``:
the MMVQ kernel tables (one translation unit per GGUF type, compiled in parallel),
the C-ABI layer with the Q8_1 quantiser and chain executor, and the C++ smithy loader.
Its entry points are declared in ``include/anvil.h``.

There is no fallback: if the library is missing or does not load, every GPU op raises
``AnvilError``.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent                      # kernel-anvil_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libanvil.so"
OBJ_DIR = ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]

# Status codes (include/anvil.h enum anvil_status).
ANVIL_OK = 0
ANVIL_ERR_INVALID = -1
ANVIL_ERR_UNSUPPORTED = -2
ANVIL_ERR_CUDA = -3
ANVIL_ERR_ALIGN = -4
ANVIL_ERR_TIMEOUT = -5
ANVIL_FLAG_PDL = 1

_STATUS_NAMES = {
    ANVIL_ERR_INVALID: "invalid argument",
    ANVIL_ERR_UNSUPPORTED: "unsupported",
    ANVIL_ERR_CUDA: "CUDA error",
    ANVIL_ERR_ALIGN: "misaligned pointer",
    ANVIL_ERR_TIMEOUT: "device wait timed out",
}


class AnvilError(RuntimeError):
    """A libanvil entry point returned a negative status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise AnvilError(ANVIL_ERR_UNSUPPORTED, "nvcc not found; cannot build libanvil.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _local_deps(src: Path) -> set[Path]:
    """src and every csrc/ or include/ header it includes, transitively (quoted includes)."""
    import re

    seen, todo = set(), [src]
    while todo:
        f = todo.pop()
        if f in seen or not f.exists():
            continue
        seen.add(f)
        for name in re.findall(r'^\s*#\s*include\s+"([^"]+)"', f.read_text(), flags=re.M):
            for d in (f.parent, CSRC, INCLUDE):
                if (d / name).exists():
                    todo.append(d / name)
                    break
    return seen


def _obj(src: Path) -> Path:
    return OBJ_DIR / (src.name + ".o")


def _stale(src: Path) -> bool:
    obj = _obj(src)
    return not obj.exists() or obj.stat().st_mtime <= max(p.stat().st_mtime for p in _local_deps(src))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    if OBJ_DIR.exists():  # a source tree with its objects: per-unit dependencies
        return any(_stale(p) or _obj(p).stat().st_mtime > t for p in _sources())
    return any(p.stat().st_mtime > t for p in _sources() + _headers())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile csrc/ into kernel_anvil/_lib/libanvil.so for sm_100a (no GPU needed)."""
    if not force and not needs_build():
        return LIB_PATH
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    inc = ["-I", str(INCLUDE), "-I", str(CSRC)]

    def compile_one(src: Path) -> Path:
        obj = _obj(src)
        if not force and not _stale(src):
            return obj  # up to date
        if src.suffix == ".cu":
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *inc, "-c", str(src), "-o", str(obj)]
        else:
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-Wall", *inc, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise AnvilError(ANVIL_ERR_UNSUPPORTED, f"compile failed: {src.name}\n{r.stderr[-4000:]}")
        return obj

    srcs = _sources()
    with ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise AnvilError(ANVIL_ERR_UNSUPPORTED, f"link failed\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None
_lib_lock = threading.Lock()

c_int, c_void_p, c_char_p, c_int64, c_uint = (
    ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int64, ctypes.c_uint)
_PI = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes); must match include/anvil.h.
SIGNATURES = {
    "anvil_abi_version": (c_int, []),
    "anvil_last_error": (c_char_p, []),
    "anvil_type_geometry": (c_int, [c_int, _PI, _PI]),
    "anvil_row_bytes": (c_int64, [c_int, c_int]),
    "anvil_quantize_q8_1": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "anvil_quantize_q8_1_ex": (c_int, [c_void_p, c_void_p, c_int, c_int, c_uint, c_void_p]),
    "anvil_mmvq": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                           c_void_p]),
    "anvil_mmvq_ex": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                              c_uint, c_void_p]),
    "anvil_mmvq_f32": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                               c_int, c_int, c_void_p]),
    "anvil_mmvq_f32_ex": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                  c_int, c_int, c_uint, c_void_p]),
    "anvil_mmvq_f32_noalloc": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                       c_int, c_int, c_void_p]),
    "anvil_mmvq_grouped": (c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                   c_int, c_int, c_uint, c_void_p]),
    "anvil_mmvq_grouped_f32": (c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int, c_int, c_int, c_int, c_uint, c_void_p]),
    "anvil_chain_add_mmvq_grouped_f32": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                                 c_void_p, c_void_p, c_int, c_int, c_int, c_int]),
    "anvil_chain_add_mmvq_grouped": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                             c_void_p, c_int, c_int, c_int, c_int]),
    "anvil_mmvq_glu": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                               c_uint, c_void_p]),
    "anvil_mmvq_glu_f32": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                   c_int, c_int, c_uint, c_void_p]),
    "anvil_chain_add_mmvq_glu": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                         c_int, c_int, c_int]),
    "anvil_take_device_status": (c_int, []),
    "anvil_mmvq_block_sums": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                      c_int, c_void_p]),
    "anvil_mmvq_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _PI, _PI, _PI, _PI]),
    "anvil_mmvq_kernel_attributes": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, _PI, _PI, _PI]),
    "anvil_chain_create": (c_void_p, []),
    "anvil_chain_destroy": (None, [c_void_p]),
    "anvil_chain_add_quantize": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "anvil_chain_add_mmvq": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                     c_int, c_int, c_int]),
    "anvil_chain_add_mmvq_f32": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_int, c_int, c_int, c_int, c_int]),
    "anvil_chain_set_coresident": (c_int, [c_void_p, c_int]),
    "anvil_chain_instantiate": (c_int, [c_void_p, c_int, c_void_p]),
    "anvil_chain_launch": (c_int, [c_void_p, c_void_p]),
    "anvil_chain_num_steps": (c_int, [c_void_p]),
    "anvil_pchain_create": (c_void_p, [c_int, c_int]),
    "anvil_pchain_destroy": (None, [c_void_p]),
    "anvil_pchain_add_group": (c_int, [c_void_p, c_void_p, c_int, c_int]),
    "anvil_pchain_add_group_chained": (c_int, [c_void_p, c_int]),
    "anvil_pchain_add_gemv": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_int]),
    "anvil_pchain_add_glu": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                                     c_int]),
    "anvil_pchain_set_group_dump": (c_int, [c_void_p, c_int, c_void_p]),
    "anvil_pchain_set_static_share": (c_int, [c_void_p, c_int]),
    "anvil_set_tensor_core_min_cols": (c_int, [c_int]),
    "anvil_get_tensor_core_min_cols": (c_int, []),
    "anvil_pchain_instantiate": (c_int, [c_void_p, c_int, c_int]),
    "anvil_pchain_set_trace": (c_int, [c_void_p, c_void_p]),
    "anvil_pchain_launch": (c_int, [c_void_p, c_void_p]),
    "anvil_pchain_epoch": (c_int, [c_void_p]),
    "anvil_pchain_read_output": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "anvil_pchain_info": (c_int, [c_void_p, _PI, _PI, _PI, _PI, _PI]),
    "anvil_pchain_gemv_shape": (c_int, [c_void_p, c_int, _PI, _PI]),
    "anvil_pchain_take_status": (c_int, []),
    "anvil_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "anvil_get_wait_limit_ns": (ctypes.c_ulonglong, []),
    "anvil_ipc_alloc": (c_int, [ctypes.c_size_t, ctypes.POINTER(c_void_p), c_void_p]),
    "anvil_ipc_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "anvil_ipc_close": (c_int, [c_void_p]),
    "anvil_ipc_free": (c_int, [c_void_p]),
    "anvil_smithy_bucket": (c_int, [c_int]),
    "anvil_smithy_set_model": (None, [c_char_p]),
    "anvil_smithy_load": (c_int, [c_char_p]),
    "anvil_smithy_try_load": (c_int, []),
    "anvil_smithy_lookup": (c_int, [c_int, c_int, c_int, _PI, _PI]),
    "anvil_smithy_reset": (None, []),
}


def lib() -> ctypes.CDLL:
    """The loaded libanvil.so (built first if sources are newer and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if needs_build():
            if LIB_PATH.exists() and shutil.which("nvcc") is None:
                pass  # prebuilt library shipped without a toolchain: use it as is
            else:
                build()
        if not LIB_PATH.exists():
            raise AnvilError(ANVIL_ERR_UNSUPPORTED, f"{LIB_PATH} is missing; run kernel_anvil._native.build()")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
        return _lib


def last_error() -> str:
    msg = lib().anvil_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(status: int) -> int:
    """Raise AnvilError for a negative status, else return it."""
    if status < 0:
        raise AnvilError(status, last_error())
    return status
