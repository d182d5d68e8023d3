"""Persistent chain: one cooperative launch per token (include/anvil.h anvil_pchain_*).

``PersistentChain`` mirrors ``mmvq.Chain`` but runs the whole token in one kernel: groups
of GEMVs that share an fp32 input (quantised to Q8_1 inside the kernel), a grid barrier
where a group depends on the ones before it, and a weight stream that never drains
between GEMVs.  With world > 1 each rank owns a row shard of every matrix and writes its
output rows straight into every rank's full output buffer (CUDA IPC peer mappings over
NVLink): the all-gather of a row-sharded GEMV fused into its epilogue.

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


class PersistentChain:
    """Builder and launcher of one persistent chain (see module docstring).

    Tensors and pointers passed in must stay valid for the chain's lifetime.
    """

    def __init__(self, world: int = 1, rank: int = 0):
        self._lib = _native.lib()
        self._h = self._lib.anvil_pchain_create(world, rank)
        if not self._h:
            raise AnvilError(_native.ANVIL_ERR_INVALID, _native.last_error())
        self.world, self.rank = world, rank
        self._keep: list = []
        self.n_gemv = 0
        self.n_groups = 0
        self.algorithmic_bytes = 0

    def add_group(self, x: torch.Tensor, wait: bool = True) -> None:
        """Start a group reading fp32 x of shape (ncols, K) or (K,)."""
        if not (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.float32
                and x.is_contiguous()):
            raise AnvilError(_native.ANVIL_ERR_INVALID, "x must be a contiguous fp32 CUDA tensor")
        x2 = x.reshape(1, -1) if x.dim() == 1 else x
        ncols, K = x2.shape
        check(self._lib.anvil_pchain_add_group(self._h, x2.data_ptr(), K, ncols, 1 if wait else 0))
        self._keep.append(x)
        self.n_groups += 1
        self._K, self._ncols = K, ncols

    def add_gemv(self, W: torch.Tensor, qt, y_ptrs, nrows: int, row0: int = 0,
                 nrows_full: int | None = None, rows_per_block: int = 0) -> None:
        """A GEMV of the current group: this rank's rows [row0, row0 + nrows) in W; y_ptrs
        is one output tensor (world 1) or each rank's full output address."""
        info = resolve_type(qt)
        if not (isinstance(W, torch.Tensor) and W.is_cuda and W.dtype == torch.uint8):
            raise AnvilError(_native.ANVIL_ERR_INVALID, "W must be a uint8 CUDA tensor")
        if isinstance(y_ptrs, torch.Tensor):
            self._keep.append(y_ptrs)
            y_ptrs = [y_ptrs.data_ptr()]
        if len(y_ptrs) != self.world:
            raise AnvilError(_native.ANVIL_ERR_INVALID, f"need {self.world} output pointers")
        nrows_full = nrows if nrows_full is None else nrows_full
        arr = (ctypes.c_void_p * MAX_RANKS)(*y_ptrs)
        check(self._lib.anvil_pchain_add_gemv(self._h, info.ggml_type, W.data_ptr(), nrows, row0,
                                              nrows_full, arr, rows_per_block))
        self._keep.append(W)
        self.n_gemv += 1
        self.algorithmic_bytes += gemv_bytes(info, nrows, self._K, self._ncols)

    def set_counters(self, ptrs: list[int]) -> None:
        arr = (ctypes.c_void_p * MAX_RANKS)(*ptrs)
        check(self._lib.anvil_pchain_set_counters(self._h, arr))

    def instantiate(self, nwarps: int = 0, ctas_per_sm: int = 0) -> None:
        check(self._lib.anvil_pchain_instantiate(self._h, nwarps, ctas_per_sm))

    def launch(self, stream: torch.cuda.Stream | None = None) -> None:
        s = stream if stream is not None else torch.cuda.current_stream()
        check(self._lib.anvil_pchain_launch(self._h, s.cuda_stream))

    def info(self) -> dict:
        v = [ctypes.c_int() for _ in range(5)]
        check(self._lib.anvil_pchain_info(self._h, *[ctypes.byref(a) for a in v]))
        return dict(zip(("grid", "nwarps", "ring_bytes", "smem_bytes", "groups"), (a.value for a in v)))

    def gemv_shape(self, index: int) -> tuple[int, int]:
        """(rows per tile, lanes per row) chosen for GEMV `index`."""
        r, lb = ctypes.c_int(), ctypes.c_int()
        check(self._lib.anvil_pchain_gemv_shape(self._h, index, ctypes.byref(r), ctypes.byref(lb)))
        return r.value, lb.value

    def close(self) -> None:
        if self._h:
            self._lib.anvil_pchain_destroy(self._h)
            self._h = None
            self._keep.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def take_status() -> int:
    """OR of the persistent kernel's device status flags since the last call
    (1 = a weight copy wait gave up, 2 = a grid barrier wait gave up)."""
    return check(_native.lib().anvil_pchain_take_status())
