"""Persistent chain: one cooperative launch per token (include/anvil.h anvil_pchain_*).

``PersistentChain`` runs a decoder token's GEMVs in one kernel: groups of GEMVs that share an
input, quantised to Q8_1 inside the kernel.  A group's input is a fixed fp32 vector or the
output of an earlier GEMV of the chain (``add_group_chained``), scaled by a power of two;
every output value is an 8-byte word {fp32 value, epoch} that is its own ready flag, so a
group waits only for the values it reads, with no grid barrier.  With world > 1 each rank
owns a row shard of every matrix and writes its output rows into every rank's output buffer
(CUDA IPC peer mappings over NVLink): the all-gather of a row-sharded GEMV inside its
epilogue.

``PeerArena`` is the shared memory for that: one device buffer per rank, exported with
CUDA IPC, opened by every other rank, carved into named regions at the same offsets on
every rank.
"""
from __future__ import annotations

import ctypes

import torch

from kernel_anvil import _native
from kernel_anvil._native import AnvilError, check
from kernel_anvil.quants import gemv_bytes, resolve_type

MAX_RANKS = 8
_IPC_HANDLE_BYTES = 64


class _DevView:
    """A raw device range as a torch tensor (via __cuda_array_interface__)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_tensor(ptr: int, shape: tuple[int, ...], dtype=torch.float32) -> torch.Tensor:
    """A torch view of device memory this library allocated (no copy, no ownership)."""
    typestr = {torch.float32: "<f4", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
    t = torch.as_tensor(_DevView(ptr, shape, typestr), device="cuda")
    if t.data_ptr() != ptr:
        raise AnvilError(_native.ANVIL_ERR_INVALID, "device view did not map in place")
    return t


class PeerArena:
    """Per-rank device buffers that every rank of a process group can read and write.

    ``layout`` is a list of (name, nbytes); each region is 256-byte aligned at the same
    offset on every rank.  ``ptrs(name)`` gives that region's address on each rank (this
    process's mapping of the peers' buffers).  Collective: every rank calls it together.
    """

    def __init__(self, layout: list[tuple[str, int]], dist, group=None):
        self._lib = _native.lib()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise AnvilError(_native.ANVIL_ERR_UNSUPPORTED, f"at most {MAX_RANKS} ranks")
        self.offsets: dict[str, int] = {}
        off = 0
        for name, nbytes in layout:
            self.offsets[name] = off
            off += (int(nbytes) + 255) & ~255
        self.nbytes = max(off, 256)
        base = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _IPC_HANDLE_BYTES)()
        check(self._lib.anvil_ipc_alloc(self.nbytes, ctypes.byref(base), handle))
        self.local = base.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        for q in range(self.world):
            if q == self.rank:
                self.bases.append(self.local)
                continue
            h = (ctypes.c_ubyte * _IPC_HANDLE_BYTES).from_buffer_copy(handles[q])
            p = ctypes.c_void_p()
            check(self._lib.anvil_ipc_open(h, ctypes.byref(p)))
            self.bases.append(p.value)
            self._opened.append(p.value)
        dist.barrier(group=group)

    def ptrs(self, name: str) -> list[int]:
        off = self.offsets[name]
        return [b + off for b in self.bases]

    def local_tensor(self, name: str, shape: tuple[int, ...], dtype=torch.float32) -> torch.Tensor:
        return device_tensor(self.local + self.offsets[name], shape, dtype)

    def close(self) -> None:
        for p in self._opened:
            self._lib.anvil_ipc_close(p)
        self._opened.clear()
        if self.local:
            self._lib.anvil_ipc_free(self.local)
            self.local = None


def output_words_bytes(nrows_full: int, ncols: int = 1) -> int:
    """Bytes of one GEMV's output buffer: two epochs of ncols x nrows_full 8-byte words."""
    return 2 * ncols * nrows_full * 8


class PersistentChain:
    """Builder and launcher of one persistent chain (see module docstring).

    Tensors and pointers passed in must stay valid for the chain's lifetime.  Indices
    returned by ``add_gemv`` / ``add_glu`` name GEMVs for ``add_group_chained`` and
    ``output``.
    """

    def __init__(self, world: int = 1, rank: int = 0):
        self._lib = _native.lib()
        self._h = self._lib.anvil_pchain_create(world, rank)
        if not self._h:
            raise AnvilError(_native.ANVIL_ERR_INVALID, _native.last_error())
        self.world, self.rank = world, rank
        self._keep: list = []
        self.n_gemv = 0
        self.algorithmic_bytes = 0
        self.ncols = 0
        self._K = 0
        self._rows_full: list[int] = []
        self._trace = None

    def add_group(self, x: torch.Tensor) -> int:
        """Start a group reading fixed fp32 x of shape (ncols, K) or (K,); returns its index."""
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32
                and x.is_contiguous()):
            raise AnvilError(_native.ANVIL_ERR_INVALID, "x must be a contiguous fp32 CUDA tensor")
        x2 = x.reshape(1, -1) if x.dim() == 1 else x
        ncols, K = x2.shape
        g = check(self._lib.anvil_pchain_add_group(self._h, x2.data_ptr(), K, ncols))
        self._keep.append(x)
        self._K, self.ncols = K, ncols
        return g

    def add_group_chained(self, src: int) -> int:
        """Start a group whose input is GEMV `src`'s output (scaled by a power of two)."""
        g = check(self._lib.anvil_pchain_add_group_chained(self._h, src))
        self._K = self._rows_full[src]
        return g

    def _ys(self, y_ptrs):
        if y_ptrs is None:
            if self.world > 1:
                raise AnvilError(_native.ANVIL_ERR_INVALID, "world > 1 needs every rank's output buffer")
            return None
        if len(y_ptrs) != self.world:
            raise AnvilError(_native.ANVIL_ERR_INVALID, f"need {self.world} output pointers")
        return (ctypes.c_void_p * MAX_RANKS)(*y_ptrs)

    def add_gemv(self, W: torch.Tensor, qt, nrows: int, row0: int = 0, nrows_full: int | None = None,
                 y_ptrs=None, rows_per_block: int = 0) -> int:
        """A GEMV of the current group: this rank's rows [row0, row0 + nrows) in W; y_ptrs is
        each rank's output buffer address (None with world 1: the chain allocates it)."""
        info = resolve_type(qt)
        if not (isinstance(W, torch.Tensor) and W.is_cuda and W.dtype == torch.uint8):
            raise AnvilError(_native.ANVIL_ERR_INVALID, "W must be a uint8 CUDA tensor")
        nrows_full = nrows if nrows_full is None else nrows_full
        idx = check(self._lib.anvil_pchain_add_gemv(self._h, info.ggml_type, W.data_ptr(), nrows, row0,
                                                    nrows_full, self._ys(y_ptrs), rows_per_block))
        self._keep.append(W)
        self._rows_full.append(nrows_full)
        self.n_gemv += 1
        self.algorithmic_bytes += gemv_bytes(info, nrows, self._K, self.ncols)
        return idx

    def add_glu(self, W_gate: torch.Tensor, W_up: torch.Tensor, qt, nrows: int, row0: int = 0,
                nrows_full: int | None = None, y_ptrs=None, rows_per_block: int = 0) -> int:
        """A gate/up pair of the current group: output row r = silu(gate[r] . x) * (up[r] . x)."""
        info = resolve_type(qt)
        for W in (W_gate, W_up):
            if not (isinstance(W, torch.Tensor) and W.is_cuda and W.dtype == torch.uint8):
                raise AnvilError(_native.ANVIL_ERR_INVALID, "weights must be uint8 CUDA tensors")
        nrows_full = nrows if nrows_full is None else nrows_full
        idx = check(self._lib.anvil_pchain_add_glu(self._h, info.ggml_type, W_gate.data_ptr(),
                                                   W_up.data_ptr(), nrows, row0, nrows_full,
                                                   self._ys(y_ptrs), rows_per_block))
        self._keep += [W_gate, W_up]
        self._rows_full.append(nrows_full)
        self.n_gemv += 1
        # two weight streams, one activation read, one output vector
        self.algorithmic_bytes += (2 * gemv_bytes(info, nrows, self._K, self.ncols)
                                   - 4 * nrows * self.ncols
                                   - gemv_bytes(info, 0, self._K, self.ncols))
        return idx

    def set_group_dump(self, group: int, out: torch.Tensor) -> None:
        """Parity probe: the staged Q8_1 blocks of `group` are written to `out` (uint8)."""
        check(self._lib.anvil_pchain_set_group_dump(self._h, group, out.data_ptr()))
        self._keep.append(out)

    def set_static_share(self, percent: int) -> None:
        """Share of each group's tiles dealt round-robin (the rest are claimed at run time)."""
        check(self._lib.anvil_pchain_set_static_share(self._h, int(percent)))

    def instantiate(self, nwarps: int = 0, ctas_per_sm: int = 0) -> None:
        check(self._lib.anvil_pchain_instantiate(self._h, nwarps, ctas_per_sm))

    def enable_trace(self) -> torch.Tensor:
        """Per CTA and group {start, staged, done, valid} %globaltimer stamps of later launches."""
        info = self.info()
        t = torch.zeros((info["grid"], info["groups"], 4), dtype=torch.int64, device="cuda")
        check(self._lib.anvil_pchain_set_trace(self._h, t.data_ptr()))
        self._trace = t
        return t

    def launch(self, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        check(self._lib.anvil_pchain_launch(self._h, s.cuda_stream))

    @property
    def epoch(self) -> int:
        return check(self._lib.anvil_pchain_epoch(self._h))

    def output(self, index: int, out: torch.Tensor | None = None,
               stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """GEMV `index`'s output of the last launch on this rank, (ncols, nrows_full) fp32
        in row order; NaN where a value did not arrive."""
        n = self._rows_full[index]
        if out is None:
            out = torch.empty((self.ncols, n), dtype=torch.float32, device="cuda")
        s = stream if stream is not None else torch.cuda.current_stream()
        check(self._lib.anvil_pchain_read_output(self._h, index, out.data_ptr(), s.cuda_stream))
        return out

    def info(self) -> dict:
        v = [ctypes.c_int() for _ in range(5)]
        check(self._lib.anvil_pchain_info(self._h, *[ctypes.byref(a) for a in v]))
        return dict(zip(("grid", "nwarps", "ring_bytes", "smem_bytes", "groups"), (a.value for a in v)))

    def gemv_shape(self, index: int) -> tuple[int, int]:
        """(rows per stage, lanes per row) chosen for GEMV `index`."""
        r, lb = ctypes.c_int(), ctypes.c_int()
        check(self._lib.anvil_pchain_gemv_shape(self._h, index, ctypes.byref(r), ctypes.byref(lb)))
        return r.value, lb.value

    def close(self) -> None:
        if self._h:
            self._lib.anvil_pchain_destroy(self._h)
            self._h = None
            self._keep.clear()
            self._trace = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def trace_summary(trace: torch.Tensor) -> list[dict]:
    """Per group over the CTAs (µs from the launch's first stamp): when warp 0 starts and ends
    its staging share (first / last CTA), when the CTAs pass the staging barrier, when warp 0
    finishes its tiles."""
    t = trace.cpu().double()
    t0 = float(t[:, 0, 0].min())
    out = []
    for g in range(t.shape[1]):
        st, se, sb, td = ((t[:, g, k] - t0) / 1e3 for k in range(4))
        out.append({"stage_start": [round(float(st.min()), 2), round(float(st.max()), 2)],
                    "stage_end": [round(float(se.min()), 2), round(float(se.max()), 2)],
                    "staged": [round(float(sb.min()), 2), round(float(sb.max()), 2)],
                    "tiles_done": [round(float(td.min()), 2), round(float(td.max()), 2)]})
    return out


def raise_on_status(status: int) -> None:
    """AnvilError(ANVIL_ERR_TIMEOUT) when a status read by take_status reports a wait that
    gave up (the launch's outputs are then wrong)."""
    if status & 3:
        what = []
        if status & 2:
            what.append("an input word did not arrive")
        if status & 1:
            what.append("a weight copy did not land")
        raise AnvilError(_native.ANVIL_ERR_TIMEOUT, "; ".join(what) + " within the wait limit")


def set_wait_limit_ns(ns: int) -> None:
    """Bound on every device-side wait of later launches (0 = the default 2 s)."""
    check(_native.lib().anvil_set_wait_limit_ns(int(ns)))


def take_status() -> int:
    """OR of the persistent kernel's device status flags since the last call
    (1 = a weight copy wait gave up, 2 = an input word did not arrive in time)."""
    return check(_native.lib().anvil_pchain_take_status())
