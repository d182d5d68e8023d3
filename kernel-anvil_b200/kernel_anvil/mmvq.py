"""Torch-facing MMVQ ops over the libanvil C ABI (include/anvil.h).

Tensors are passed as raw device pointers together with torch's current CUDA stream, so
the ops compose with torch code and with CUDA graph capture.  All ops require CUDA
tensors: there is no CPU path.

Layouts (GGUF / llama.cpp conventions):
  W   uint8 (nrows, row_bytes): row r holds K/qk consecutive blocks of the quant type.
  x   fp32 (ncols, K): ncols activation columns.
  xq  uint8 (ncols, K/32*36): Q8_1 blocks {half d, half s, int8 q[32]} per column.
  y   fp32 (ncols, nrows).
"""
from __future__ import annotations

import ctypes

import torch

from kernel_anvil import _native
from kernel_anvil._native import ANVIL_FLAG_PDL, AnvilError, check
from kernel_anvil.quants import Q8_1_BLOCK_SIZE, QuantTypeInfo, resolve_type

MAX_COLS = 8
MAX_SEGMENTS = 4  # matrices of one grouped launch


def _stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(name: str, t: torch.Tensor, dtype: torch.dtype) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise AnvilError(_native.ANVIL_ERR_INVALID, f"{name} must be a CUDA tensor (no CPU path)")
    if t.dtype != dtype:
        raise AnvilError(_native.ANVIL_ERR_INVALID, f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise AnvilError(_native.ANVIL_ERR_INVALID, f"{name} must be contiguous")


def q8_1_bytes(K: int, ncols: int = 1) -> int:
    return ncols * (K // 32) * Q8_1_BLOCK_SIZE


def quantize_q8_1(x: torch.Tensor, out: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """Quantise fp32 activations (ncols, K) or (K,) to Q8_1 blocks (llama.cpp quantize_q8_1)."""
    _require_cuda("x", x, torch.float32)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    ncols, K = x2.shape
    if out is None:
        out = torch.empty((ncols, q8_1_bytes(K)), dtype=torch.uint8, device=x.device)
    _require_cuda("out", out, torch.uint8)
    if out.numel() < q8_1_bytes(K, ncols):
        raise AnvilError(_native.ANVIL_ERR_INVALID, "out is too small")
    check(_native.lib().anvil_quantize_q8_1_ex(x2.data_ptr(), out.data_ptr(), K, ncols,
                                               ANVIL_FLAG_PDL if pdl else 0, _stream_ptr()))
    return out


def _shape_args(W: torch.Tensor, info: QuantTypeInfo, nrows, K):
    if W.dim() == 2:
        nrows = W.shape[0] if nrows is None else nrows
        if K is None:
            if W.shape[1] % info.block_size:
                raise AnvilError(_native.ANVIL_ERR_INVALID, "row bytes not a multiple of the block size")
            K = W.shape[1] // info.block_size * info.qk
    if nrows is None or K is None:
        raise AnvilError(_native.ANVIL_ERR_INVALID, "nrows and K are needed for a flat W")
    if W.numel() < nrows * info.row_bytes(K):
        raise AnvilError(_native.ANVIL_ERR_INVALID, "W is smaller than nrows x row_bytes")
    return nrows, K


def mmvq(W: torch.Tensor, qt, xq: torch.Tensor, nrows: int | None = None, K: int | None = None,
         ncols: int | None = None, nwarps: int = 0, rows_per_block: int = 0,
         out: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """y = W @ dequant(xq) for ncols Q8_1 columns: the sm_100a MMVQ kernel.

    nwarps / rows_per_block of 0 use the smithy table entry for (type, nrows, K) or the
    built-in default.  ``pdl=True`` lets the kernel prefetch W before the previous kernel
    in the stream finishes (W must not be produced by that kernel).
    """
    info = resolve_type(qt)
    _require_cuda("W", W, torch.uint8)
    _require_cuda("xq", xq, torch.uint8)
    nrows, K = _shape_args(W, info, nrows, K)
    if ncols is None:
        ncols = xq.numel() // q8_1_bytes(K)
    if not 1 <= ncols <= MAX_COLS:
        raise AnvilError(_native.ANVIL_ERR_INVALID, f"ncols={ncols} outside 1..{MAX_COLS}")
    if xq.numel() < q8_1_bytes(K, ncols):
        raise AnvilError(_native.ANVIL_ERR_INVALID, "xq is too small")
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=W.device)
    _require_cuda("out", out, torch.float32)
    if out.numel() < ncols * nrows:
        raise AnvilError(_native.ANVIL_ERR_INVALID, "out is too small")
    check(_native.lib().anvil_mmvq_ex(info.ggml_type, W.data_ptr(), xq.data_ptr(), out.data_ptr(),
                                      nrows, K, ncols, nwarps, rows_per_block,
                                      ANVIL_FLAG_PDL if pdl else 0, _stream_ptr()))
    return out


def mmvq_f32(W: torch.Tensor, qt, x: torch.Tensor, nwarps: int = 0, rows_per_block: int = 0,
             xq_scratch: torch.Tensor | None = None, out: torch.Tensor | None = None,
             pdl: bool = False) -> torch.Tensor:
    """y = W @ dequant(Q8_1(x)) from fp32 x (ncols, K), as llama.cpp's MMVQ path computes it.

    One kernel quantises x in its prologue when it fits (else quantise + MMVQ); the result
    is bit-identical to quantize_q8_1 followed by mmvq."""
    info = resolve_type(qt)
    _require_cuda("W", W, torch.uint8)
    _require_cuda("x", x, torch.float32)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    ncols, K = x2.shape
    nrows, K = _shape_args(W, info, None, K)
    if xq_scratch is None:
        xq_scratch = torch.empty(q8_1_bytes(K, ncols), dtype=torch.uint8, device=W.device)
    _require_cuda("xq_scratch", xq_scratch, torch.uint8)
    if out is None:
        out = torch.empty((ncols, nrows), dtype=torch.float32, device=W.device)
    _require_cuda("out", out, torch.float32)
    check(_native.lib().anvil_mmvq_f32_ex(info.ggml_type, W.data_ptr(), x2.data_ptr(),
                                          xq_scratch.data_ptr(), out.data_ptr(), nrows, K, ncols,
                                          nwarps, rows_per_block, ANVIL_FLAG_PDL if pdl else 0,
                                          _stream_ptr()))
    return out


def _seg_arrays(Ws, ys, nrows):
    n = len(Ws)
    if not 1 <= n <= MAX_SEGMENTS or len(ys) != n or len(nrows) != n:
        raise AnvilError(_native.ANVIL_ERR_INVALID, f"1..{MAX_SEGMENTS} matrices with one output each")
    return ((ctypes.c_void_p * n)(*[w.data_ptr() for w in Ws]),
            (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys]),
            (ctypes.c_int * n)(*nrows))


def mmvq_grouped_f32(Ws: list, qt, x: torch.Tensor, nwarps: int = 0, rows_per_block: int = 0,
                     xq_scratch: torch.Tensor | None = None, outs: list | None = None,
                     pdl: bool = False) -> list:
    """[W @ dequant(Q8_1(x)) for W in Ws] in one launch: matrices of one quant type reading the
    same fp32 x (ncols, K).  Each output equals mmvq_f32(W, qt, x) alone."""
    info = resolve_type(qt)
    _require_cuda("x", x, torch.float32)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    ncols, K = x2.shape
    rows = []
    for W in Ws:
        _require_cuda("W", W, torch.uint8)
        rows.append(_shape_args(W, info, None, K)[0])
    if xq_scratch is None:
        xq_scratch = torch.empty(q8_1_bytes(K, ncols), dtype=torch.uint8, device=x.device)
    if outs is None:
        outs = [torch.empty((ncols, n), dtype=torch.float32, device=x.device) for n in rows]
    for y in outs:
        _require_cuda("out", y, torch.float32)
    Wa, ya, ra = _seg_arrays(Ws, outs, rows)
    check(_native.lib().anvil_mmvq_grouped_f32(info.ggml_type, len(Ws), Wa, x2.data_ptr(),
                                               xq_scratch.data_ptr(), ya, ra, K, ncols, nwarps,
                                               rows_per_block, ANVIL_FLAG_PDL if pdl else 0,
                                               _stream_ptr()))
    return outs


def _glu_shapes(W_gate: torch.Tensor, W_up: torch.Tensor, info: QuantTypeInfo, K: int) -> int:
    _require_cuda("W_gate", W_gate, torch.uint8)
    _require_cuda("W_up", W_up, torch.uint8)
    nrows = _shape_args(W_gate, info, None, K)[0]
    if _shape_args(W_up, info, None, K)[0] != nrows:
        raise AnvilError(_native.ANVIL_ERR_INVALID, "gate and up need the same number of rows")
    return nrows


def mmvq_glu(W_gate: torch.Tensor, W_up: torch.Tensor, qt, xq: torch.Tensor, nwarps: int = 0,
             rows_per_block: int = 0, out: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """silu(W_gate @ dequant(xq)) * (W_up @ dequant(xq)) for one Q8_1 column, in one launch.

    Each product is what mmvq computes for its matrix; neither is written out.  Rows of
    W_gate / W_up must be a multiple of 16 bytes."""
    info = resolve_type(qt)
    _require_cuda("xq", xq, torch.uint8)
    K = W_gate.shape[1] // info.block_size * info.qk
    nrows = _glu_shapes(W_gate, W_up, info, K)
    if xq.numel() < q8_1_bytes(K):
        raise AnvilError(_native.ANVIL_ERR_INVALID, "xq is too small")
    if out is None:
        out = torch.empty((1, nrows), dtype=torch.float32, device=xq.device)
    _require_cuda("out", out, torch.float32)
    if out.numel() < nrows:
        raise AnvilError(_native.ANVIL_ERR_INVALID, "out is too small")
    check(_native.lib().anvil_mmvq_glu(info.ggml_type, W_gate.data_ptr(), W_up.data_ptr(), xq.data_ptr(),
                                       out.data_ptr(), nrows, K, nwarps, rows_per_block,
                                       ANVIL_FLAG_PDL if pdl else 0, _stream_ptr()))
    return out


def mmvq_glu_f32(W_gate: torch.Tensor, W_up: torch.Tensor, qt, x: torch.Tensor, nwarps: int = 0,
                 rows_per_block: int = 0, xq_scratch: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, pdl: bool = False) -> torch.Tensor:
    """mmvq_glu from fp32 x (K values): quantise to Q8_1, then the gate/up launch."""
    info = resolve_type(qt)
    _require_cuda("x", x, torch.float32)
    K = x.numel()
    nrows = _glu_shapes(W_gate, W_up, info, K)
    if xq_scratch is None:
        xq_scratch = torch.empty(q8_1_bytes(K), dtype=torch.uint8, device=x.device)
    _require_cuda("xq_scratch", xq_scratch, torch.uint8)
    if out is None:
        out = torch.empty((1, nrows), dtype=torch.float32, device=x.device)
    _require_cuda("out", out, torch.float32)
    if xq_scratch.numel() < q8_1_bytes(K) or out.numel() < nrows:
        raise AnvilError(_native.ANVIL_ERR_INVALID, "xq_scratch or out is too small")
    check(_native.lib().anvil_mmvq_glu_f32(info.ggml_type, W_gate.data_ptr(), W_up.data_ptr(),
                                           x.contiguous().data_ptr(), xq_scratch.data_ptr(),
                                           out.data_ptr(), nrows, K, nwarps, rows_per_block,
                                           ANVIL_FLAG_PDL if pdl else 0, _stream_ptr()))
    return out


def block_sums(W: torch.Tensor, qt, xq: torch.Tensor, nrows: int | None = None, K: int | None = None,
               ncols: int | None = None, nwarps: int = 0, rows_per_block: int = 0) -> torch.Tensor:
    """The production kernel's exact int32 block dots, shape (ncols, nrows, nsub).

    nsub = K/16 for the types with 16-weight scale groups (Q6_K, Q2_K, Q3_K, IQ2_XS, IQ2_S,
    IQ1_M), K/32 otherwise (one per Q8_1 block).
    """
    info = resolve_type(qt)
    _require_cuda("W", W, torch.uint8)
    _require_cuda("xq", xq, torch.uint8)
    nrows, K = _shape_args(W, info, nrows, K)
    if ncols is None:
        ncols = xq.numel() // q8_1_bytes(K)
    nsub = K // 16 if info.name in ("Q6_K", "Q2_K", "Q3_K", "IQ2_XS", "IQ2_S", "IQ1_M") else K // 32
    out = torch.empty((ncols, nrows, nsub), dtype=torch.int32, device=W.device)
    check(_native.lib().anvil_mmvq_block_sums(info.ggml_type, W.data_ptr(), xq.data_ptr(),
                                              out.data_ptr(), nrows, K, ncols, nwarps,
                                              rows_per_block, _stream_ptr()))
    return out


def host_lanes_per_row(nblk: int, rpb: int) -> int:
    """Lanes per row the single-GEMV kernel uses for rows of nblk blocks in tiles of rpb
    rows (the twin of host_lanes_per_row in csrc/mmvq.cuh): the power of two that keeps the
    most lanes busy, preferring more lanes on ties."""
    best, best_u, lb = 32, -1.0, 32
    while lb >= 1:
        per_lane = -(-nblk // lb)
        u = nblk / (lb * per_lane) * min(rpb / (32 // lb), 1.0)
        if u > best_u + 1e-6:
            best, best_u = lb, u
        lb //= 2
    return best


def plan(qt, nrows: int, K: int, ncols: int = 1, nwarps: int = 0, rows_per_block: int = 0) -> dict:
    """Launch geometry the library would use: nwarps, rows_per_block, grid, smem bytes."""
    info = resolve_type(qt)
    v = [ctypes.c_int() for _ in range(4)]
    check(_native.lib().anvil_mmvq_plan(info.ggml_type, nrows, K, ncols, nwarps, rows_per_block,
                                        *[ctypes.byref(a) for a in v]))
    return {"nwarps": v[0].value, "rows_per_block": v[1].value, "grid": v[2].value,
            "smem_bytes": v[3].value}


def kernel_attributes(qt, nrows: int, K: int, ncols: int = 1, nwarps: int = 0,
                      rows_per_block: int = 0) -> dict:
    """Compiled resources of the kernel that plan() would launch: registers per thread, local
    (spill) bytes per thread, maximum threads per block (cudaFuncGetAttributes)."""
    info = resolve_type(qt)
    v = [ctypes.c_int() for _ in range(3)]
    check(_native.lib().anvil_mmvq_kernel_attributes(info.ggml_type, nrows, K, ncols, nwarps,
                                                     rows_per_block, *[ctypes.byref(a) for a in v]))
    return {"regs_per_thread": v[0].value, "local_bytes": v[1].value, "max_threads_per_block": v[2].value}


def set_tensor_core_min_cols(min_cols: int) -> None:
    """Q4_K / Q5_K launches with at least min_cols columns (2..8) and no explicit launch shape
    use the mma.sync tensor-core kernel; 0 turns it off (every launch on the dp4a kernels)."""
    check(_native.lib().anvil_set_tensor_core_min_cols(int(min_cols)))


def tensor_core_min_cols() -> int:
    return int(_native.lib().anvil_get_tensor_core_min_cols())


class tensor_cores:
    """Context manager: `with tensor_cores(0): ...` runs the block on the dp4a kernels."""

    def __init__(self, min_cols: int):
        self.min_cols = min_cols

    def __enter__(self):
        self.saved = tensor_core_min_cols()
        set_tensor_core_min_cols(self.min_cols)
        return self

    def __exit__(self, *exc):
        set_tensor_core_min_cols(self.saved)
        return False


def take_device_status() -> int:
    """OR of device status flags raised since the last call (1 = an mbarrier wait gave up)."""
    return check(_native.lib().anvil_take_device_status())


class Chain:
    """An ordered list of quantize / MMVQ steps on fixed buffers, captured once into a CUDA
    graph (native executor, include/anvil.h anvil_chain_*) and replayed per token.

    The tensors passed to ``add_*`` must stay alive (and at the same address) for the
    chain's lifetime; the chain keeps references to them.
    """

    def __init__(self):
        self._lib = _native.lib()
        self._h = self._lib.anvil_chain_create()
        if not self._h:
            raise AnvilError(_native.ANVIL_ERR_CUDA, "anvil_chain_create failed")
        self._keep: list[torch.Tensor] = []
        self.instantiated = False
        self.weight_bytes = 0
        self.algorithmic_bytes = 0
        self.n_mmvq = 0
        self.n_quantize = 0
        self.n_launches = 0

    def add_quantize(self, x: torch.Tensor, xq: torch.Tensor) -> None:
        _require_cuda("x", x, torch.float32)
        _require_cuda("xq", xq, torch.uint8)
        x2 = x.reshape(1, -1) if x.dim() == 1 else x
        ncols, K = x2.shape
        if xq.numel() < q8_1_bytes(K, ncols):
            raise AnvilError(_native.ANVIL_ERR_INVALID, "xq is too small")
        check(self._lib.anvil_chain_add_quantize(self._h, x2.data_ptr(), xq.data_ptr(), K, ncols))
        self._keep += [x, xq]
        self.n_quantize += 1
        self.n_launches += 1

    def add_mmvq(self, W: torch.Tensor, qt, xq: torch.Tensor, y: torch.Tensor, nrows: int | None = None,
                 K: int | None = None, ncols: int = 1, nwarps: int = 0, rows_per_block: int = 0) -> None:
        info = resolve_type(qt)
        _require_cuda("W", W, torch.uint8)
        _require_cuda("xq", xq, torch.uint8)
        _require_cuda("y", y, torch.float32)
        nrows, K = _shape_args(W, info, nrows, K)
        if xq.numel() < q8_1_bytes(K, ncols) or y.numel() < ncols * nrows:
            raise AnvilError(_native.ANVIL_ERR_INVALID, "xq or y is too small")
        check(self._lib.anvil_chain_add_mmvq(self._h, info.ggml_type, W.data_ptr(), xq.data_ptr(),
                                             y.data_ptr(), nrows, K, ncols, nwarps, rows_per_block))
        self._keep += [W, xq, y]
        self.n_mmvq += 1
        self.n_launches += 1
        self.weight_bytes += nrows * info.row_bytes(K)
        from kernel_anvil.quants import gemv_bytes
        self.algorithmic_bytes += gemv_bytes(info, nrows, K, ncols)

    def add_mmvq_f32(self, W: torch.Tensor, qt, x: torch.Tensor, xq_scratch: torch.Tensor,
                     y: torch.Tensor, nrows: int | None = None, K: int | None = None, ncols: int = 1,
                     nwarps: int = 0, rows_per_block: int = 0) -> None:
        """GEMV step from fp32 x (quantisation fused into the GEMV when it fits)."""
        info = resolve_type(qt)
        _require_cuda("W", W, torch.uint8)
        _require_cuda("x", x, torch.float32)
        _require_cuda("xq_scratch", xq_scratch, torch.uint8)
        _require_cuda("y", y, torch.float32)
        nrows, K = _shape_args(W, info, nrows, K)
        if x.numel() < K * ncols or xq_scratch.numel() < q8_1_bytes(K, ncols) or y.numel() < ncols * nrows:
            raise AnvilError(_native.ANVIL_ERR_INVALID, "x, xq_scratch or y is too small")
        check(self._lib.anvil_chain_add_mmvq_f32(self._h, info.ggml_type, W.data_ptr(), x.data_ptr(),
                                                 xq_scratch.data_ptr(), y.data_ptr(), nrows, K, ncols,
                                                 nwarps, rows_per_block))
        self._keep += [W, x, xq_scratch, y]
        self.n_mmvq += 1
        self.n_launches += 1
        self.weight_bytes += nrows * info.row_bytes(K)
        from kernel_anvil.quants import gemv_bytes
        self.algorithmic_bytes += gemv_bytes(info, nrows, K, ncols)

    def add_mmvq_grouped(self, Ws: list, qt, xq: torch.Tensor, ys: list, nrows: list, K: int,
                         ncols: int = 1, nwarps: int = 0, rows_per_block: int = 0) -> None:
        """One launch for several GEMVs of type qt reading the Q8_1 activation xq."""
        info = resolve_type(qt)
        _require_cuda("xq", xq, torch.uint8)
        if xq.numel() < q8_1_bytes(K, ncols):
            raise AnvilError(_native.ANVIL_ERR_INVALID, "xq is too small")
        for W, y, n in zip(Ws, ys, nrows):
            _require_cuda("W", W, torch.uint8)
            _require_cuda("y", y, torch.float32)
            if W.numel() < n * info.row_bytes(K) or y.numel() < ncols * n:
                raise AnvilError(_native.ANVIL_ERR_INVALID, "W or y is too small")
        Wa, ya, ra = _seg_arrays(Ws, ys, nrows)
        check(self._lib.anvil_chain_add_mmvq_grouped(self._h, info.ggml_type, len(Ws), Wa,
                                                     xq.data_ptr(), ya, ra, K, ncols, nwarps,
                                                     rows_per_block))
        self._keep += [*Ws, xq, *ys]
        from kernel_anvil.quants import gemv_bytes
        for n in nrows:
            self.n_mmvq += 1
            self.weight_bytes += n * info.row_bytes(K)
            self.algorithmic_bytes += gemv_bytes(info, n, K, ncols)
        self.n_launches += 1

    def add_mmvq_grouped_f32(self, Ws: list, qt, x: torch.Tensor, xq_scratch: torch.Tensor, ys: list,
                             nrows: list, K: int, ncols: int = 1, nwarps: int = 0,
                             rows_per_block: int = 0) -> None:
        """One launch for several GEMVs of type qt reading fp32 x (see mmvq_grouped_f32)."""
        info = resolve_type(qt)
        _require_cuda("x", x, torch.float32)
        _require_cuda("xq_scratch", xq_scratch, torch.uint8)
        for W, y, n in zip(Ws, ys, nrows):
            _require_cuda("W", W, torch.uint8)
            _require_cuda("y", y, torch.float32)
            if W.numel() < n * info.row_bytes(K) or y.numel() < ncols * n:
                raise AnvilError(_native.ANVIL_ERR_INVALID, "W or y is too small")
        Wa, ya, ra = _seg_arrays(Ws, ys, nrows)
        check(self._lib.anvil_chain_add_mmvq_grouped_f32(self._h, info.ggml_type, len(Ws), Wa,
                                                         x.data_ptr(), xq_scratch.data_ptr(), ya, ra,
                                                         K, ncols, nwarps, rows_per_block))
        self._keep += [*Ws, x, xq_scratch, *ys]
        from kernel_anvil.quants import gemv_bytes
        for n in nrows:
            self.n_mmvq += 1
            self.weight_bytes += n * info.row_bytes(K)
            self.algorithmic_bytes += gemv_bytes(info, n, K, ncols)
        self.n_launches += 1

    def add_mmvq_glu(self, W_gate: torch.Tensor, W_up: torch.Tensor, qt, xq: torch.Tensor,
                     y: torch.Tensor, nwarps: int = 0, rows_per_block: int = 0) -> None:
        """One launch: y = silu(W_gate @ dequant(xq)) * (W_up @ dequant(xq)), one column."""
        info = resolve_type(qt)
        _require_cuda("xq", xq, torch.uint8)
        _require_cuda("y", y, torch.float32)
        K = W_gate.shape[1] // info.block_size * info.qk
        nrows = _glu_shapes(W_gate, W_up, info, K)
        if xq.numel() < q8_1_bytes(K) or y.numel() < nrows:
            raise AnvilError(_native.ANVIL_ERR_INVALID, "xq or y is too small")
        check(self._lib.anvil_chain_add_mmvq_glu(self._h, info.ggml_type, W_gate.data_ptr(),
                                                 W_up.data_ptr(), xq.data_ptr(), y.data_ptr(), nrows,
                                                 K, nwarps, rows_per_block))
        self._keep += [W_gate, W_up, xq, y]
        from kernel_anvil.quants import gemv_bytes
        self.n_mmvq += 2
        self.weight_bytes += 2 * nrows * info.row_bytes(K)
        # both matrices and one read of xq; one output row of 4 bytes per gate/up pair
        self.algorithmic_bytes += 2 * gemv_bytes(info, nrows, K, 1) - nrows * 4 - q8_1_bytes(K)
        self.n_launches += 1

    def set_coresident(self, kernels_per_sm: int) -> None:
        """Size GEMV grids so that this many consecutive GEMVs fit on each SM together."""
        check(self._lib.anvil_chain_set_coresident(self._h, kernels_per_sm))

    def instantiate(self, pdl: bool = True, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        check(self._lib.anvil_chain_instantiate(self._h, 1 if pdl else 0, s.cuda_stream))
        self.instantiated = True

    def launch(self, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        check(self._lib.anvil_chain_launch(self._h, s.cuda_stream))

    @property
    def num_steps(self) -> int:
        return self._lib.anvil_chain_num_steps(self._h)

    def close(self) -> None:
        if self._h:
            self._lib.anvil_chain_destroy(self._h)
            self._h = None
            self._keep.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
