"""ctypes wrapper of the CPU oracle (oracle/anvil_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the checker,
and by bench.py's cpu_baseline / reference leg.  The product (kernel-anvil_b200/) never
imports it.  Every function here is a thin call into the C restatement; see the C file's
header for the reference file:line each piece follows.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
REF_SMITHY = HERE / "_ref" / "libsmithy_ref.so"

TYPE_IDS = {"Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12,
            "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ2_XS": 17, "IQ3_XXS": 18, "IQ1_S": 19,
            "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "IQ1_M": 29}
# types with one block sum per 16 weights (their scale groups); the others one per 32
SUB16_IDS = (10, 11, 14, 17, 22, 29)

_lib = None


def build() -> None:
    """make -C oracle (liboracle.so, plus oracle/_ref when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "anvil_oracle.c").stat().st_mtime:
            build()
        h = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        h.oracle_quantize_q8_1.argtypes = [P, P, I64, I64]
        h.oracle_quantize_q8_1_chained.argtypes = [P, P, P, I64, I64]
        h.oracle_mmvq_d32.argtypes = [ctypes.c_int, P, P, P, I64, I64, I64]
        h.oracle_dequant.argtypes = [ctypes.c_int, P, P, I64, I64]
        h.oracle_block_sums.argtypes = [ctypes.c_int, P, P, P, I64, I64, I64]
        h.oracle_mmvq.argtypes = [ctypes.c_int, P, P, P, I64, I64, I64]
        h.oracle_float_to_half.argtypes = [ctypes.c_float]
        h.oracle_float_to_half.restype = ctypes.c_uint16
        h.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        h.oracle_half_to_float.restype = ctypes.c_float
        h.oracle_num_threads.restype = ctypes.c_int
        h.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _lib = h
    return _lib


def _tid(qt) -> int:
    return qt if isinstance(qt, int) else TYPE_IDS[qt]


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    """x (ncols, K) fp32 -> (ncols, K/32*36) uint8 Q8_1 blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
    ncols, K = x.shape
    out = np.empty((ncols, K // 32 * 36), dtype=np.uint8)
    lib().oracle_quantize_q8_1(_ptr(x), _ptr(out), K, ncols)
    return out


def quantize_q8_1_chained(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The persistent chain's chained-input quantisation of x (ncols, K): Q8_1-shaped blocks
    with the quants of quantize_q8_1 and d in fp32 (bytes 0-3), and per column the power of
    two 2^-e (e = exponent of the column's max |x|) that the GEMV applies to its result."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
    ncols, K = x.shape
    out = np.empty((ncols, K // 32 * 36), dtype=np.uint8)
    scale = np.empty(ncols, dtype=np.float32)
    lib().oracle_quantize_q8_1_chained(_ptr(x), _ptr(out), _ptr(scale), K, ncols)
    return out, scale


def mmvq_chained(qt, W: np.ndarray, xq: np.ndarray, scale: np.ndarray, nrows: int, K: int,
                 ncols: int = 1) -> np.ndarray:
    """y (ncols, nrows) float64 of a chained group: the block formula with fp32 d8, times the
    column's scale."""
    out = np.empty((ncols, nrows), dtype=np.float64)
    W = np.ascontiguousarray(W, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    if lib().oracle_mmvq_d32(_tid(qt), _ptr(W), _ptr(xq), _ptr(out), nrows, K, ncols) != 0:
        raise ValueError("bad type or K")
    return out * np.asarray(scale, dtype=np.float64).reshape(ncols, 1)


def mmvq_glu_chained(qt, W_gate: np.ndarray, W_up: np.ndarray, xq: np.ndarray, scale: np.ndarray,
                     nrows: int, K: int) -> np.ndarray:
    """silu(g) * u (1, nrows) float64 of a chained gate/up pair (g, u scaled first)."""
    g = mmvq_chained(qt, W_gate, xq, scale, nrows, K)
    u = mmvq_chained(qt, W_up, xq, scale, nrows, K)
    return g / (1.0 + np.exp(-g)) * u


def dequantize(qt, W: np.ndarray, nrows: int, K: int) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint8)
    out = np.empty((nrows, K), dtype=np.float32)
    if lib().oracle_dequant(_tid(qt), _ptr(W), _ptr(out), nrows, K) != 0:
        raise ValueError("bad type or K")
    return out


def dequantize_q8_1(xq: np.ndarray, K: int) -> np.ndarray:
    """Q8_1 blocks -> fp32 values d * q (the dequantised activation a dot product sees)."""
    blocks = np.ascontiguousarray(xq, dtype=np.uint8).reshape(-1, 36)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)
    q = blocks[:, 4:36].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1, K)


def block_sums(qt, W: np.ndarray, xq: np.ndarray, nrows: int, K: int, ncols: int = 1) -> np.ndarray:
    nsub = K // 16 if _tid(qt) in SUB16_IDS else K // 32
    out = np.empty((ncols, nrows, nsub), dtype=np.int32)
    W = np.ascontiguousarray(W, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    if lib().oracle_block_sums(_tid(qt), _ptr(W), _ptr(xq), _ptr(out), nrows, K, ncols) != 0:
        raise ValueError("bad type or K")
    return out


def mmvq(qt, W: np.ndarray, xq: np.ndarray, nrows: int, K: int, ncols: int = 1) -> np.ndarray:
    """y (ncols, nrows) float64 from exact block sums."""
    out = np.empty((ncols, nrows), dtype=np.float64)
    W = np.ascontiguousarray(W, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    if lib().oracle_mmvq(_tid(qt), _ptr(W), _ptr(xq), _ptr(out), nrows, K, ncols) != 0:
        raise ValueError("bad type or K")
    return out


def mmvq_glu(qt, W_gate: np.ndarray, W_up: np.ndarray, xq: np.ndarray, nrows: int, K: int) -> np.ndarray:
    """silu(y_gate) * y_up (1, nrows) float64: the SwiGLU product that follows the gate and up
    GEMVs of a llama.cpp decode step (ggml GLU, silu(g) = g / (1 + exp(-g)): the "GLU | silu +
    elementwise mul" op of docs/vulkan-vs-rocm-analysis.md:135, fused after the gate GEMV as
    "Q4_K fused (gate+SiLU)" in docs/decode-pipeline-breakdown.md:40)."""
    g = mmvq(qt, W_gate, xq, nrows, K)
    u = mmvq(qt, W_up, xq, nrows, K)
    return g / (1.0 + np.exp(-g)) * u


def float_to_half_bits(v: float) -> int:
    return int(lib().oracle_float_to_half(v))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(n)


def max_rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max |y - ref| / max |ref| -- the normalised error the parity tolerance is stated in."""
    ref = np.asarray(ref, dtype=np.float64)
    scale = float(np.max(np.abs(ref))) or 1.0
    return float(np.max(np.abs(np.asarray(y, dtype=np.float64) - ref)) / scale)


# ---- the reference's own smithy loader (oracle/_ref, compiled from its header) ------

_ref = None


def ref_smithy():
    """ctypes handle of oracle/_ref/libsmithy_ref.so, or None when it was not built."""
    global _ref
    if _ref is None:
        if not REF_SMITHY.exists():
            try:
                build()
            except Exception:
                return None
        if not REF_SMITHY.exists():
            return None
        h = ctypes.CDLL(str(REF_SMITHY))
        PI = ctypes.POINTER(ctypes.c_int)
        h.ref_smithy_bucket.argtypes = [ctypes.c_int]
        h.ref_smithy_set_model.argtypes = [ctypes.c_char_p]
        h.ref_smithy_load.argtypes = [ctypes.c_char_p]
        h.ref_smithy_lookup.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, PI, PI]
        h.ref_smithy_cell.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, PI, PI]
        _ref = h
    return _ref
