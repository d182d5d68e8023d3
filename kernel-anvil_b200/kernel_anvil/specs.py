"""NVIDIA B200 hardware constants and an occupancy model (replaces the reference's AMD
table, kernel_anvil/rdna3.py:8-210, with the same GpuSpec / detect_gpu / HEURISTICS surface).

Bandwidth: ``peak_bandwidth_gbs`` is the measured HBM copy bandwidth of this pool when
MEASURED_PEAKS.json is present (6537.3 GB/s when written), else 6650 GB/s;
``nominal_bandwidth_gbs`` is the 8 TB/s data-sheet figure.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path


def _measured_hbm() -> float:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except Exception:
        return 6650.0


@dataclass(frozen=True)
class GpuSpec:
    name: str
    arch: str
    peak_bandwidth_gbs: float
    nominal_bandwidth_gbs: float
    sm_count: int
    max_warps_per_sm: int
    max_blocks_per_sm: int
    regs_per_sm: int
    reg_alloc_unit: int       # registers per warp are allocated in units of this many
    max_regs_per_thread: int
    smem_per_sm_bytes: int
    smem_per_block_bytes: int
    smem_reserved_per_block: int
    l2_bytes: int
    wave_size: int = 32

    @property
    def gfx(self) -> str:
        """Architecture tag (the reference's field name)."""
        return self.arch

    def max_reg_warps(self, regs_per_thread: int) -> int:
        if regs_per_thread <= 0:
            return self.max_warps_per_sm
        per_warp = -(-regs_per_thread * self.wave_size // self.reg_alloc_unit) * self.reg_alloc_unit
        return min(self.max_warps_per_sm, self.regs_per_sm // per_warp)

    def max_smem_blocks(self, smem_bytes: int) -> int:
        if smem_bytes <= 0:
            return self.max_blocks_per_sm
        return self.smem_per_sm_bytes // (smem_bytes + self.smem_reserved_per_block)

    def occupancy(self, regs_per_thread: int, smem_bytes: int, threads_per_block: int) -> tuple[float, str]:
        """(active warps as % of the SM maximum, limiting resource)."""
        wpb = -(-threads_per_block // self.wave_size)
        by_regs = self.max_reg_warps(regs_per_thread) // wpb
        by_smem = self.max_smem_blocks(smem_bytes)
        by_warps = self.max_warps_per_sm // wpb
        blocks = min(by_regs, by_smem, by_warps, self.max_blocks_per_sm)
        pct = 100.0 * blocks * wpb / self.max_warps_per_sm
        lim = min((by_regs, "regs"), (by_smem, "smem"), (by_warps, "warps"),
                  (self.max_blocks_per_sm, "blocks"))[1]
        return pct, lim


B200 = GpuSpec(
    name="NVIDIA B200", arch="sm_100a",
    peak_bandwidth_gbs=_measured_hbm(), nominal_bandwidth_gbs=8000.0,
    sm_count=148, max_warps_per_sm=64, max_blocks_per_sm=32,
    regs_per_sm=65536, reg_alloc_unit=256, max_regs_per_thread=255,
    smem_per_sm_bytes=228 * 1024, smem_per_block_bytes=227 * 1024, smem_reserved_per_block=1024,
    l2_bytes=126 * 1024 * 1024,
)

GPU_SPECS = {"sm_100a": B200, "sm_100": B200}


def detect_gpu() -> GpuSpec | None:
    """B200 when torch sees a compute-capability 10.0 device (or one named B200)."""
    try:
        import torch

        if torch.cuda.is_available():
            name = torch.cuda.get_device_name(0)
            if torch.cuda.get_device_capability(0) == (10, 0) or "B200" in name:
                return B200
    except Exception:
        pass
    return None


HEURISTICS = [
    "A decode GEMV moves ~0.56 B per weight (Q4_K) and does 2 flops: it is HBM bound",
    "Keep >= 32 KB of weight loads in flight per SM (bandwidth x latency) to saturate HBM",
    "Stream weight tiles with bulk async copies into shared memory; no registers are tied up",
    "Stage the Q8_1 activation once per CTA; persistent CTAs amortise it over many rows",
    "Inside a chain, start the next GEMV's weight stream before its dependency wait (PDL)",
    "Rotate weight buffers past the 126 MB L2 when timing, or the numbers measure L2",
    "Shared-memory reads of 16-byte chunks must cover distinct bank quads per quarter warp",
]
